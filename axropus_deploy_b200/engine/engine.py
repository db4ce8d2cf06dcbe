"""Serving engine: continuous batching over a paged KV cache with AMF restore.

One engine per GPU. Each :meth:`LLMEngine.step`:

1. **Admission.** Waiting requests are admitted while blocks and the prefill token
   budget allow. For each: the live prefix cache (G2) is matched block by block;
   the rest of the page-aligned prefix is looked up in the AMF tiers; a hit is
   restored straight into freshly allocated blocks by the page-transfer kernel
   (pull + dequantise + scatter, over NVLink when the owning shard is another GPU)
   and the restored blocks are registered in the prefix cache as computed.
2. **Prefill** of every admitted request's uncomputed tokens (restored or cached
   pages are skipped), one varlen batch; cold prefixes are then captured into the G1
   tier (quantise + push to the owner shard).
3. **Decode** of all running requests, one token each (split-KV attention over the
   pages, bf16/FP8/INT4). Optional CUDA graphs replay the decode step.

Reference: the AMF state machine of the native engine (core/engine.cpp:2607-3120)
and the vLLM connector path (korith_vllm_ext/amf_kv_connector.py), where restore
and save are per-layer PyTorch index-puts synchronous with the forward pass.
"""
from __future__ import annotations

import contextlib
import itertools
import logging
import os
import time
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .. import ops
from ..amf.manager import AmfHit, AmfManager
from ..models.llama import AttnMeta, LlamaModel
from ..ops.kvcache import PAGE, KVCache
from .block_manager import BlockManager, block_hashes

log = logging.getLogger(__name__)


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    stop_token_ids: Sequence[int] = ()
    seed: Optional[int] = None


@dataclass
class Request:
    req_id: str
    prompt: List[int]
    params: SamplingParams
    amf_prefix_len: Optional[int] = None
    blocks: List[int] = field(default_factory=list)
    num_computed: int = 0
    output: List[int] = field(default_factory=list)
    state: str = "waiting"
    t_arrival: float = 0.0
    t_admit: float = 0.0
    t_first_token: float = 0.0
    t_finish: float = 0.0
    amf_tier: str = "cold"
    local_cached_tokens: int = 0
    restored_tokens: int = 0
    restore_ms: float = 0.0
    row: int = -1
    prompt_np: Optional[np.ndarray] = None
    hashes: List[bytes] = field(default_factory=list)
    prefill_start: int = 0   # first prompt position this engine computed itself (after any reuse)
    prefill_end: int = 0     # end of the part of the prompt the current step prefills

    @property
    def ttft_ms(self) -> float:
        return (self.t_first_token - self.t_arrival) * 1e3

    @property
    def seq_len(self) -> int:
        return len(self.prompt) + len(self.output)


@dataclass
class EngineConfig:
    num_blocks: int = 1024
    kv_fmt: str = "bf16"
    max_batch: int = 64
    max_prefill_tokens: int = 16384
    max_model_len: int = 32768
    enable_prefix_cache: bool = True
    capture_on_miss: bool = True
    amf_min_tokens: int = 64
    cuda_graphs: bool = False
    # with cuda_graphs: one-sequence prefills of <= 512 new tokens (AMF-hit suffixes) replay
    # CUDA graphs too (dense single-GPU models)
    prefill_graphs: bool = True
    # expert parallelism: every GPU runs exactly one prefill and one decode forward per
    # step (empty when it has nothing to do) so the MoE collectives of all GPUs line up
    lockstep: bool = False
    # speculative decoding of greedy requests: "" (off), "ngram" (prompt lookup), "model"
    # (needs a draft model) or "pool" (several drafters, each sequence's distinct drafts
    # verified together on copy-on-write KV branches); depth adapts between 1 and
    # spec_max_depth
    spec: str = ""
    spec_max_depth: int = 8
    # [AMF_*] trace lines (None: KORITH_AMF_TRACE decides)
    trace: Optional[bool] = None
    # shared-prefix decode: running sequences whose block tables start with the same
    # (prefix-cache / AMF-restored) pages attend to them in one grouped pass per step;
    # groups need at least this many shared pages. Off (0) by default: at the headline
    # shape (32 x 8.4 K tokens, Zipf prefix reuse) the plain split-KV decode already reads
    # shared pages about once, because the CTAs of sequences that share them run together
    # and hit in L2 (0.127 ms per layer plain against 0.237 ms grouped, measured on B200)
    cascade_min_pages: int = 0
    # greedy CUDA-graph decode launches step t + 1 before it reads step t's tokens
    pipeline_decode: bool = True
    # a step that admits prompts while others decode runs both in one forward (the decode
    # rows ride along the prefill's projections instead of streaming the weights again)
    mixed_batch: bool = True
    # with mixed steps: while other sequences decode, a step prefills at most this many
    # new prompt tokens (a long prompt continues over several steps, and the decoding
    # sequences advance in each: shorter inter-token gaps during long cold prefills);
    # 0 prefills whole prompts. Off by default: at the headline workload whole prompts
    # gave 2911 output tok/s against 2848 with 2048-token chunks and 2676 with 1024
    prefill_chunk: int = 0


_NVTX = os.environ.get("AXR_NVTX", "0") == "1"


@contextlib.contextmanager
def _nvtx(name: str):
    """NVTX range around an engine phase when AXR_NVTX=1 (for nsys / ncu range filters)."""
    if _NVTX and torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


class LLMEngine:
    def __init__(self, model: LlamaModel, cfg: EngineConfig, amf: Optional[AmfManager] = None, draft_model=None):
        self.model = model
        self.cfg = cfg
        self.amf = amf
        if hasattr(model, "ensure_positions"):
            model.ensure_positions(cfg.max_model_len + PAGE)
        mc = model.cfg
        self.device = model.device
        kv_heads = getattr(model, "cache_kv_heads", mc.num_kv_heads)  # tensor parallel: this GPU's heads
        self.cache = KVCache(model.num_layers, cfg.num_blocks, kv_heads, mc.head_dim, cfg.kv_fmt, self.device)
        self._agree = getattr(model, "agree_min", None)
        self.bm = BlockManager(cfg.num_blocks, cfg.enable_prefix_cache)
        self.max_blocks_per_seq = (cfg.max_model_len + PAGE - 1) // PAGE
        self.block_table = torch.zeros(cfg.max_batch, self.max_blocks_per_seq, dtype=torch.int32, device=self.device)
        self.free_rows = list(range(cfg.max_batch - 1, -1, -1))
        self.waiting: List[Request] = []
        self.running: List[Request] = []
        self.finished: List[Request] = []
        self._ids = itertools.count()
        self._graphs = None
        self._pin: Optional[torch.Tensor] = None  # pinned staging buffer of step inputs
        self._pin_ev = None                        # recorded after the last copy out of it
        if cfg.cuda_graphs and self.device.type == "cuda" and not model.cfg.is_moe:
            from .cuda_graph import DecodeGraphRunner

            self._graphs = DecodeGraphRunner(self)
        self._prefill_graphs = None
        if cfg.cuda_graphs and cfg.prefill_graphs and self.device.type == "cuda" and type(model) is LlamaModel \
                and not model.cfg.is_moe:
            from .cuda_graph import PrefillGraphRunner

            self._prefill_graphs = PrefillGraphRunner(self)
        from .scheduler import AdmissionPolicy
        from .trace import AmfTrace

        self.policy = AdmissionPolicy()
        if getattr(model, "agree_min", None) is not None:
            # tensor-parallel ranks must admit identically; their pool views may differ
            self.policy.enabled = False

        self.trace = AmfTrace(cfg.trace)
        self.spec = None
        if cfg.spec:
            from .spec import ModelDrafter, SpecDecoder

            if cfg.spec == "model":
                if draft_model is None:
                    raise ValueError("spec='model' needs a draft_model")
                if hasattr(draft_model, "ensure_positions"):
                    draft_model.ensure_positions(cfg.max_model_len + PAGE)
                drafter = ModelDrafter(draft_model, cfg.num_blocks)
            elif cfg.spec in ("ngram", "pool"):
                drafter = None
            else:
                raise ValueError(f"unknown spec mode {cfg.spec!r}")
            if cfg.spec == "pool":
                # a pool of draft engines (n-gram lookups of several lengths, plus the draft
                # model when one is given); each sequence's distinct proposals are verified
                # together on copy-on-write KV branches
                from .pool import DraftPool, PoolSpecDecoder
                from .spec import NgramDrafter

                drafters = [NgramDrafter(3, 1), NgramDrafter(3, 1, skip=1), NgramDrafter(6, 4)]
                if draft_model is not None:
                    if hasattr(draft_model, "ensure_positions"):
                        draft_model.ensure_positions(cfg.max_model_len + PAGE)
                    drafters.insert(0, ModelDrafter(draft_model, cfg.num_blocks))
                self.spec = PoolSpecDecoder(self, cfg.spec_max_depth, DraftPool(drafters))
            else:
                self.spec = SpecDecoder(self, cfg.spec_max_depth, drafter)
        self.stat = {"steps": 0, "prefill_tokens": 0, "decode_tokens": 0, "restored_tokens": 0,
                     "local_cached_tokens": 0, "cold_prefill_tokens": 0, "cascade_steps": 0,
                     "cascade_grouped_seqs": 0, "pipelined_decode_steps": 0, "sync_wait_ms": 0.0, "mixed_steps": 0,
                     "chunked_prefills": 0}
        # decode pipelining: a greedy graph decode launched but whose tokens are not read yet
        self._pipe: Optional[dict] = None
        from ..ops.attention import cascade_supported

        self._cascade_on = (cfg.cascade_min_pages > 0 and self.device.type == "cuda" and
                            cascade_supported(self.cache, mc.head_dim) and type(model) is LlamaModel)
        self._casc_key = None
        self._casc_plan = None
        self._casc_serial = itertools.count(1)

    # ------------------------------------------------------------------ API
    def add_request(self, prompt: Sequence[int], params: Optional[SamplingParams] = None, req_id: Optional[str] = None,
                    amf_prefix_len: Optional[int] = None, arrival: Optional[float] = None) -> Request:
        params = params or SamplingParams()
        if len(prompt) + params.max_tokens > self.cfg.max_model_len:
            raise ValueError("prompt + max_tokens exceeds max_model_len")
        arr = np.asarray(prompt, dtype=np.int64)
        r = Request(req_id or f"req-{next(self._ids)}", arr.tolist(), params, amf_prefix_len)
        r.prompt_np = (arr & 0xFFFFFFFF).astype(np.uint32).view(np.int32)
        r.t_arrival = arrival if arrival is not None else time.perf_counter()
        self.waiting.append(r)
        return r

    def has_unfinished(self) -> bool:
        return bool(self.waiting or self.running or self._pipe is not None)

    def generate(self, prompts: Sequence[Sequence[int]], params: Optional[SamplingParams] = None) -> List[List[int]]:
        reqs = [self.add_request(p, params) for p in prompts]
        while self.has_unfinished():
            self.step()
        return [r.output for r in reqs]

    def generate_requests(self, prompts: Sequence[Sequence[int]], params: Optional[SamplingParams] = None,
                          amf_prefix_len: Optional[int] = None) -> List[List[int]]:
        """Public batch API: run the prompts to completion and return their tokens."""
        reqs = [self.add_request(p, params, amf_prefix_len=amf_prefix_len) for p in prompts]
        while self.has_unfinished():
            self.step()
        return [r.output for r in reqs]

    def _trace_key(self, r: Request, limit: int, hit) -> None:
        from ..amf.keys import amf_hash_tokens

        disk = getattr(self.amf, "disk", None)
        ctx = getattr(disk, "ctx", None)
        self.trace.key("hit" if hit is not None else "miss", getattr(ctx, "model_hash", 0),
                       getattr(ctx, "tenant_hash", 0), amf_hash_tokens(r.prompt[:limit]), self.cfg.max_model_len,
                       self.cfg.max_prefill_tokens, getattr(ctx, "rope_base_bits", 0),
                       getattr(ctx, "rope_scale_bits", 0), getattr(ctx, "sampling_hash", 0), getattr(ctx, "rng_hash", 0))
        if hit is None:
            r.amf_miss_reason = "first_request" if self.amf.stat.get("captures", 0) == 0 else "not_found"

    def run_summary(self) -> dict:
        """``[KORITH_RUN_SUMMARY]`` line (when tracing) and its fields."""
        gen = sum(len(r.output) for r in self.finished) + sum(len(r.output) for r in self.running)
        if self.amf is not None and self.trace.enabled:
            a = self.amf.stat
            self.trace.stats({"saved_ms": self.trace.n["saved_ms"], "saved_tokens": self.stat["restored_tokens"],
                              "hits": self.trace.n["hits"], "misses": self.trace.n["misses"],
                              "blocks": self.stat["restored_tokens"] // PAGE,
                              "failures": a.get("capture_failures", 0), "admit": a.get("captures", 0)})
        return self.trace.summary(gen)

    def warmup_graphs(self) -> int:
        """Capture the decode CUDA graph of every batch bucket now (start-up work), so no
        capture lands in the middle of serving; returns the number captured."""
        if self._graphs is None:
            return 0
        n = 0
        for b in self._graphs.buckets:
            if b not in self._graphs.graphs:
                self._graphs._capture(b)
                n += 1
        return n

    def close(self) -> None:
        """Release CUDA graphs (they hold device memory and must go before the
        process group is destroyed)."""
        if self._pipe is not None:  # let the step in flight end before its buffers go
            self._pipe["event"].synchronize()
            self._pipe = None
        if self._graphs is not None:
            self._graphs.close()
            self._graphs = None
        if self._prefill_graphs is not None:
            self._prefill_graphs.close()
            self._prefill_graphs = None
        pool = getattr(self.spec, "pool", None)
        if pool is not None:
            pool.close()

    def evict_live_cache(self, fraction: float = 1.0) -> int:
        """Drop cached (unreferenced) KV blocks -- forces later requests to restore from AMF."""
        return self.bm.evict_cached(fraction)

    # ------------------------------------------------------------------ step
    def step(self) -> List[Request]:
        self.stat["steps"] += 1
        done: List[Request] = []
        if self._pipe is not None:
            pipe = self._pipe
            in_pipe = {id(r) for r in pipe["reqs"]}
            joined = any(r.state == "running" and id(r) not in in_pipe for r in self.running)
            prefilling = any(r.state == "prefilling" for r in self.running)
            if not self.waiting and not joined and not prefilling:
                # nothing to admit and nobody new to decode: launch the next decode on the
                # device tokens of the one in flight, then read the in-flight step's tokens
                # while the GPU runs it
                cont = [r for r in pipe["reqs"] if r.state == "running" and len(r.output) + 1 < r.params.max_tokens]
                nxt = self._decode_launch(cont, pipe) if cont else None
                done += self._pipe_finish()
                self._pipe = nxt
                return done
            # requests to admit, or admitted last step (their first decode input is on the
            # host): end the pipeline for one step so the next launch batches everyone
            done += self._pipe_finish()
            self._pipe = None
        with _nvtx("admit"):
            admitted = self._admit()
        decoding = [r for r in self.running if r.state == "running" and r not in admitted]
        # prompts being prefilled in chunks continue first, then the newly admitted ones
        admitted = [r for r in self.running if r.state == "prefilling" and r not in admitted] + admitted
        admitted = self._plan_chunks(admitted, decoding)
        any_prefill, any_decode = bool(admitted), bool(decoding)
        if self.cfg.lockstep and hasattr(self.model, "ep_any"):
            # a forward runs on every GPU when it runs on any (the MoE layers need all of them)
            any_prefill, any_decode = self.model.ep_any([any_prefill, any_decode])
        if admitted and decoding and self._mixable(admitted, decoding):
            with _nvtx("mixed"):
                return done + self._mixed(admitted, decoding)
        if admitted:
            with _nvtx("prefill"):
                done += self._prefill(admitted)
        elif self.cfg.lockstep and any_prefill:
            self._idle_forward()
        if decoding:
            with _nvtx("decode"):
                if self._pipelinable(decoding):
                    self._pipe = self._decode_launch(decoding, None)
                else:
                    done += self._decode(decoding)
        elif self.cfg.lockstep and any_decode:
            self._idle_forward()
        if self.device.type == "cuda" and self._pipe is None:
            self._check_kernel_errors()
        return done

    # ------------------------------------------------------------------ decode pipelining
    def _pipelinable(self, reqs: List[Request]) -> bool:
        """Greedy CUDA-graph decode of the single-GPU model: the next step's input tokens can
        stay on the device."""
        return (self.cfg.pipeline_decode and self._graphs is not None and self.spec is None and not self.cfg.lockstep and
                type(self.model) is LlamaModel and all(r.params.temperature <= 0 for r in reqs))

    def _decode_launch(self, reqs: List[Request], prev: Optional[dict]) -> dict:
        """Launches one decode step of ``reqs``. With ``prev`` (the step in flight) each
        request's input token is the one ``prev`` is computing: it stays on the device."""
        toks, pos, slots, lens = [], [], [], []
        for r in reqs:
            p = r.seq_len if prev is not None else r.seq_len - 1  # position of the input token
            pos.append(p)
            slots.append(r.blocks[p // PAGE] * PAGE + p % PAGE)
            lens.append(p + 1)
            if prev is None:
                toks.append(r.output[-1])
        plan = self.cascade_plan(reqs)
        if plan is not None:
            self.stat["cascade_steps"] += 1
            self.stat["cascade_grouped_seqs"] += plan["grouped"]
        dev_tokens = None
        if prev is not None:
            where = {id(r): i for i, r in enumerate(prev["reqs"])}
            dev_tokens = [where[id(r)] for r in reqs]
            self.stat["pipelined_decode_steps"] += 1
        self.stat["decode_tokens"] += len(reqs)
        _, slot, ev = self._graphs.run(reqs, None if prev is not None else toks, pos, slots, lens, plan, dev_tokens)
        return {"reqs": reqs, "slot": slot, "event": ev}

    def _pipe_finish(self) -> List[Request]:
        """Waits for the step in flight, checks the kernels' error flag and appends its tokens
        (requests that finished meanwhile on a stop token drop theirs)."""
        pipe = self._pipe
        t0 = time.perf_counter()
        pipe["event"].synchronize()
        self.stat["sync_wait_ms"] += (time.perf_counter() - t0) * 1e3
        n = len(pipe["reqs"])
        vals = self._graphs.tok_host[pipe["slot"], :n + 1].tolist()
        if vals[n]:
            self._pipe = None
            raise RuntimeError(f"a fused kernel gave up waiting (error code {vals[n]}); outputs of this step are "
                               "invalid (a peer GPU stopped or fell behind by more than the wait bound)")
        done: List[Request] = []
        for r, t in zip(pipe["reqs"], vals[:n]):
            if r.state == "running":
                self._append(r, t, done)
        return done

    def _check_kernel_errors(self) -> None:
        """The tcgen05 / peer kernels record a code instead of hanging when a bounded wait
        runs out; their outputs are then incomplete, so the step must not be used."""
        from ..ops.gemm import error_flag

        code = int(error_flag(self.device)[0].item())
        if code:
            raise RuntimeError(f"a fused kernel gave up waiting (error code {code}); outputs of this step are "
                               "invalid (a peer GPU stopped or fell behind by more than the wait bound)")

    def _idle_forward(self) -> None:
        empty = torch.empty(0, dtype=torch.int32, device=self.device)
        meta = AttnMeta(mode="decode", positions=empty, slots=empty, block_table=self.block_table[:0],
                        seq_lens=empty)
        self.model.forward(empty, meta, self.cache)

    # ------------------------------------------------------------------ admission
    def _amf_limit(self, r: Request) -> int:
        lim = (len(r.prompt) - 1) // PAGE * PAGE  # keep >= 1 token to prefill
        if r.amf_prefix_len is not None:
            lim = min(lim, r.amf_prefix_len // PAGE * PAGE)
        return max(0, lim)

    def _held(self, r: Request) -> bool:
        """Is r's prefix held by the live prefix cache or a G1 tier (admission order only)?"""
        if len(r.prompt) > PAGE:
            first = block_hashes(r.prompt_np, 1)
            if first and first[0] in self.bm.by_hash:
                return True
        if self.amf is not None and self.amf.router is not None and r.amf_prefix_len:
            from ..amf.keys import pool_key

            g1 = self.amf.raw_pool or self.amf.comp_pool
            return bool(g1 is not None and g1.contains(pool_key(r.prompt[: r.amf_prefix_len // PAGE * PAGE])))
        return False

    def _admit(self) -> List[Request]:
        admitted: List[Request] = []
        if len(self.waiting) > 1:
            self.waiting = self.policy.order(self.waiting, self._held, spec=self.spec is not None)
        decoding = sum(1 for r in self.running if r.state == "running")
        head_hit = bool(self.waiting) and bool(self.waiting[0].__dict__.get("_held"))
        budget = self.policy.budget(self.cfg.max_prefill_tokens, decoding, self.cfg.max_batch, head_hit)
        budget0 = budget
        # cfg.max_batch may be lowered at run time (a batch controller); rows stay allocated for the start value
        while self.waiting and self.free_rows and len(self.running) < self.cfg.max_batch:
            r = self.waiting[0]
            limit = self._amf_limit(r)
            full_pages = (len(r.prompt) - 1) // PAGE
            hashes = block_hashes(r.prompt_np, full_pages)
            r.hashes = hashes
            matched = self.bm.match_prefix(hashes)
            n_local = len(matched)
            hit: Optional[AmfHit] = None
            if self.amf is not None and n_local * PAGE < limit:
                hit = self.amf.lookup(r.prompt_np, limit)
                if self._agree is not None:
                    # tensor parallel: every rank restores the same pages (the shortest hit)
                    n = self._agree(hit.n_pages if hit is not None else 0)
                    if hit is not None and n < hit.n_pages:
                        hit.n_tokens = n * PAGE
                if hit is not None and hit.n_pages <= n_local:
                    hit.release()
                    hit = None
                if self.trace.enabled:
                    self._trace_key(r, limit, hit)
            computed_pages = max(n_local, hit.n_pages if hit else 0)
            new_tokens = len(r.prompt) - computed_pages * PAGE
            if admitted and new_tokens > budget:
                self.bm.release(matched)
                if hit:
                    hit.release()
                break
            need = (len(r.prompt) + r.params.max_tokens + PAGE - 1) // PAGE - n_local
            if not self.bm.can_allocate(need):
                self.bm.release(matched)
                if hit:
                    hit.release()
                if not self.running and not admitted:
                    raise MemoryError("request does not fit in the KV cache")
                break
            self.waiting.pop(0)
            r.blocks = matched + self.bm.allocate(need)
            r.t_admit = time.perf_counter()
            r.local_cached_tokens = n_local * PAGE
            if hit is not None:
                t0 = time.perf_counter()
                blk = torch.tensor(r.blocks[n_local:hit.n_pages], dtype=torch.int32)
                ev = None
                if self.device.type == "cuda":
                    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    ev[0].record()
                try:
                    hit.restore(self.cache, blk, first_page=n_local)
                except BaseException:
                    hit.release()
                    raise
                r.restore_ms = (time.perf_counter() - t0) * 1e3
                if ev is not None:
                    # the restore runs on the GPU while this step builds and launches the
                    # prefill; the source entry stays pinned until the step's first
                    # synchronisation (_settle_restores), which also reads the device time
                    ev[1].record()
                    r._restore = (hit, ev)
                else:
                    hit.release()
                    self._note_restore(r, hit)
                r.restored_tokens = (hit.n_pages - n_local) * PAGE
                r.amf_tier = hit.tier
                self.bm.register_computed(r.blocks[n_local:hit.n_pages], hashes[n_local:hit.n_pages])
                if hit.tier in ("lmcache", "disk") and self.amf.promote_lmcache_hits:
                    self.amf.capture(r.prompt_np[:hit.n_tokens], self.cache,
                                     torch.tensor(r.blocks[:hit.n_pages], dtype=torch.int32),
                                     promote_from=hit.tier)
                self.stat["restored_tokens"] += r.restored_tokens
            elif n_local:
                r.amf_tier = "apc"
            r.num_computed = computed_pages * PAGE
            r.prefill_start = r.num_computed
            self.stat["local_cached_tokens"] += n_local * PAGE
            r.row = self.free_rows.pop()
            r.state = "prefilling"
            self.running.append(r)
            admitted.append(r)
            budget -= new_tokens
        self.policy.note(waiting=len(self.waiting), decoding=decoding, budget_tokens=budget0, head_is_hit=head_hit,
                         admitted=len(admitted), held_waiting=sum(1 for w in self.waiting if w.__dict__.get("_held")))
        return admitted

    def _note_restore(self, r: Request, hit) -> None:
        self.amf.note_restored(hit, r.restore_ms, 0.0)
        self.trace.hit(len(r.prompt), hit.n_tokens, hit.n_tokens, r.restore_ms, hit.tier)

    def _settle_restores(self, reqs: List[Request], ok: bool = True) -> None:
        """After the step's first synchronisation: device time of each restore, release of
        the pinned source entries, statistics and trace lines."""
        for r in reqs:
            pending = r.__dict__.pop("_restore", None)
            if pending is None:
                continue
            hit, (e0, e1) = pending
            if ok:
                r.restore_ms = e0.elapsed_time(e1)
            else:
                e1.synchronize()  # the copy must be done before its source may be reused
            hit.release()
            if ok:
                self._note_restore(r, hit)

    # ------------------------------------------------------------------ forward helpers
    def _sample(self, logits: torch.Tensor, reqs: List[Request]) -> List[int]:
        if all(r.params.temperature <= 0 for r in reqs):
            return ops.argmax(logits).tolist()
        out = ops.argmax(logits).tolist()
        for i, r in enumerate(reqs):
            if r.params.temperature > 0:
                p = torch.softmax(logits[i].float() / r.params.temperature, dim=-1)
                g = torch.Generator(device=p.device)
                g.manual_seed((r.params.seed or 0) + len(r.output))
                out[i] = int(torch.multinomial(p, 1, generator=g))
        return out

    def _append(self, r: Request, tok: int, done: List[Request]) -> None:
        now = time.perf_counter()
        if not r.output:
            r.t_first_token = now
        r.output.append(tok)
        if len(r.output) >= r.params.max_tokens or tok in r.params.stop_token_ids:
            r.state = "finished"
            r.t_finish = now
            self.running.remove(r)
            self.bm.release(r.blocks)
            self.free_rows.append(r.row)
            r.row = -1
            self.finished.append(r)
            done.append(r)

    def _set_rows(self, reqs: List[Request]) -> None:
        for r in reqs:
            row = torch.tensor(r.blocks, dtype=torch.int32)
            self.block_table[r.row, : len(r.blocks)] = row.to(self.device, non_blocking=True)

    def _stage_int32(self, *parts) -> List[torch.Tensor]:
        """Host int32 arrays -> device tensors with one copy from a reused pinned buffer.
        The buffer is rewritten only after the previous copy out of it has completed (its
        event; normally long done, since the sampling of every step synchronises)."""
        arrs = [np.asarray(p, dtype=np.int32).reshape(-1) for p in parts]
        if self.device.type != "cuda":
            return [torch.from_numpy(a.copy()) for a in arrs]
        total = sum(a.size for a in arrs)
        if self._pin_ev is not None:
            self._pin_ev.synchronize()
        if self._pin is None or self._pin.numel() < total:
            self._pin = torch.empty(max(total, 1 << 16), dtype=torch.int32, pin_memory=True)
        view = self._pin.numpy()
        off = 0
        for a in arrs:
            view[off:off + a.size] = a
            off += a.size
        dev_all = self._pin[:total].to(self.device, non_blocking=True)
        if self._pin_ev is None:
            self._pin_ev = torch.cuda.Event()
        self._pin_ev.record()
        out, off = [], 0
        for a in arrs:
            out.append(dev_all[off:off + a.size])
            off += a.size
        return out

    def _prefill_inputs(self, reqs: List[Request]):
        """Host arrays of a prefill of ``reqs``: tokens, positions, slots, cu_q, lengths and
        each request's first prefilled position."""
        toks, pos, slots, cu, lens = [], [], [], [0], []
        prefilled_from = {}
        for r in reqs:
            s, e = r.num_computed, r.prefill_end
            prefilled_from[r.req_id] = r.prefill_start
            n = e - s
            toks.extend(r.prompt[s:e])
            p = np.arange(s, e)
            pos.extend(p.tolist())
            b = np.asarray(r.blocks, dtype=np.int64)
            slots.extend((b[p // PAGE] * PAGE + p % PAGE).tolist())
            cu.append(cu[-1] + n)
            lens.append(e)
            self.stat["prefill_tokens"] += n
            if r.amf_tier == "cold":
                self.stat["cold_prefill_tokens"] += n
        return toks, pos, slots, cu, lens, prefilled_from

    def _plan_chunks(self, reqs: List[Request], decoding: List[Request]) -> List[Request]:
        """Sets each prefilling request's ``prefill_end`` for this step and returns those
        that prefill anything. While other sequences decode (mixed steps), at most
        ``cfg.prefill_chunk`` new tokens are prefilled per step, in admission order; with
        nothing decoding, or without mixed steps, whole prompts."""
        chunked = bool(decoding) and self.cfg.prefill_chunk > 0 and bool(reqs) and self._mixable(reqs, decoding)
        left = self.cfg.prefill_chunk if chunked else None
        out = []
        for r in reqs:
            rem = len(r.prompt) - r.num_computed
            take = rem if left is None else min(rem, left)
            if take <= 0:
                continue
            r.prefill_end = r.num_computed + take
            out.append(r)
            if take < rem:
                self.stat["chunked_prefills"] += 1
            if left is not None:
                left -= take
        return out

    def _prefill(self, reqs: List[Request]) -> List[Request]:
        toks, pos, slots, cu, lens, prefilled_from = self._prefill_inputs(reqs)
        self._set_rows(reqs)
        fin = [i for i, r in enumerate(reqs) if r.prefill_end == len(r.prompt)]
        t_pf = time.perf_counter()
        try:
            if (len(fin) == len(reqs) and self._prefill_graphs is not None and
                    self._prefill_graphs.supports(reqs, len(toks), lens[0])):
                logits = self._prefill_graphs.run(reqs[0], toks, pos, slots, lens[0])
            else:
                # every input of the step in one copy from pinned host memory
                d_toks, d_pos, d_slots, d_lens, d_cu, d_idx, d_rows = self._stage_int32(
                    toks, pos, slots, lens, cu, [cu[i + 1] - 1 for i in fin], [r.row for r in reqs])
                meta = AttnMeta(mode="prefill", positions=d_pos, slots=d_slots,
                                block_table=self.block_table.index_select(0, d_rows.long()), seq_lens=d_lens, cu_q=d_cu,
                                max_q=max(cu[i + 1] - cu[i] for i in range(len(reqs))), max_seq_len=max(lens),
                                logits_idx=d_idx)
                logits = self.model.forward(d_toks, meta, self.cache)
            # synchronises with the forward (and the restores); a step that only carries
            # chunks of longer prompts samples nothing and waits for the GPU here instead
            new = self._sample(logits, [reqs[i] for i in fin]) if fin else self._sync_step()
        except BaseException:
            self._settle_restores(reqs, ok=False)
            raise
        self._settle_restores(reqs)
        return self._finish_prefill(reqs, new, prefilled_from, len(toks), (time.perf_counter() - t_pf) * 1e3)

    def _sync_step(self) -> List[int]:
        if self.device.type == "cuda":
            torch.cuda.current_stream(self.device).synchronize()
        return []

    def _finish_prefill(self, reqs: List[Request], new: List[int], prefilled_from: dict, n_new: int,
                        pf_ms: float) -> List[Request]:
        """After a prefill step: prefix-cache registration of the pages computed so far; for
        the requests whose whole prompt is now computed (``new`` holds their sampled tokens,
        in order) trace lines, AMF capture of what this engine computed, first output
        tokens; the others keep prefilling in later steps."""
        fin = [r for r in reqs if r.prefill_end == len(r.prompt)]
        cold = [r for r in fin if r.amf_tier == "cold"]
        if cold and len(cold) == len(reqs):
            self.trace.note_prefill(n_new, pf_ms)
        if self.amf is not None and self.trace.enabled:
            for r in cold:
                share = (len(r.prompt) - prefilled_from[r.req_id]) / max(1, n_new)
                self.trace.miss(getattr(r, "amf_miss_reason", "first_request"), pf_ms * share, len(r.prompt))
        done: List[Request] = []
        it = iter(new)
        for r in reqs:
            r.num_computed = r.prefill_end
            full = r.num_computed // PAGE
            hs = r.hashes if len(r.hashes) >= full else block_hashes(r.prompt_np, full)
            self.bm.register_computed(r.blocks[:full], hs[:full])
            if r.num_computed < len(r.prompt):
                continue  # more chunks to come
            # capture when this engine computed a real part of the prefix itself: a cold
            # miss, or a shorter hit (G2 or AMF) that this prompt extended
            if self.amf is not None and self.cfg.capture_on_miss:
                lim = self._amf_limit(r)
                if lim >= self.cfg.amf_min_tokens and lim - prefilled_from[r.req_id] >= self.cfg.amf_min_tokens:
                    self.amf.capture(r.prompt_np[:lim], self.cache, torch.tensor(r.blocks[: lim // PAGE],
                                                                              dtype=torch.int32))
            r.state = "running"
            self._append(r, next(it), done)
        return done

    # ------------------------------------------------------------------ mixed steps
    def _mixable(self, admitted: List[Request], decoding: List[Request]) -> bool:
        """One forward for the step's prefills and decodes: the single-GPU dense model, no
        lockstep (expert parallelism), no speculative decoding."""
        return (self.cfg.mixed_batch and type(self.model) is LlamaModel and not self.cfg.lockstep and
                self.spec is None and self.model.ep is None)

    def _mixed(self, preqs: List[Request], dreqs: List[Request]) -> List[Request]:
        """Prefill of ``preqs`` and one decode step of ``dreqs`` in one forward: rows
        [0, Tp) are the prompts' new tokens, the rows after them one token per decoding
        sequence; every projection runs once over all rows, attention in two kernels."""
        toks, pos, slots, cu, lens, prefilled_from = self._prefill_inputs(preqs)
        dtoks, dpos, dslots, dlens = self.decode_meta(dreqs)
        self.stat["decode_tokens"] += len(dreqs)
        self.stat["mixed_steps"] += 1
        tp = len(toks)
        self._set_rows(preqs)
        fin = [i for i, r in enumerate(preqs) if r.prefill_end == len(r.prompt)]
        idx = [cu[i + 1] - 1 for i in fin] + list(range(tp, tp + len(dreqs)))
        t_pf = time.perf_counter()
        try:
            d_toks, d_pos, d_slots, d_lens, d_cu, d_idx, d_rows, d_dlens, d_drows = self._stage_int32(
                toks + dtoks, pos + dpos, slots + dslots, lens, cu, idx, [r.row for r in preqs], dlens,
                [r.row for r in dreqs])
            dmeta = AttnMeta(mode="decode", positions=d_pos[tp:], slots=d_slots[tp:],
                             block_table=self.block_table.index_select(0, d_drows.long()), seq_lens=d_dlens,
                             max_seq_len=max(dlens))
            meta = AttnMeta(mode="mixed", positions=d_pos, slots=d_slots,
                            block_table=self.block_table.index_select(0, d_rows.long()), seq_lens=d_lens, cu_q=d_cu,
                            max_q=max(cu[i + 1] - cu[i] for i in range(len(preqs))), max_seq_len=max(lens),
                            logits_idx=d_idx, decode=dmeta)
            logits = self.model.forward(d_toks, meta, self.cache)
            new = self._sample(logits, [preqs[i] for i in fin] + dreqs)
        except BaseException:
            self._settle_restores(preqs, ok=False)
            raise
        self._settle_restores(preqs)
        done = self._finish_prefill(preqs, new[:len(fin)], prefilled_from, tp, (time.perf_counter() - t_pf) * 1e3)
        for r, t in zip(dreqs, new[len(fin):]):
            self._append(r, t, done)
        if self.device.type == "cuda":
            self._check_kernel_errors()
        return done

    def decode_meta(self, reqs: List[Request]) -> tuple:
        toks, pos, slots, lens = [], [], [], []
        for r in reqs:
            p = r.seq_len - 1
            toks.append(r.output[-1])
            pos.append(p)
            slots.append(r.blocks[p // PAGE] * PAGE + p % PAGE)
            lens.append(p + 1)
        return toks, pos, slots, lens

    def cascade_plan(self, reqs: List[Request]) -> Optional[dict]:
        """Shared-prefix groups of a decode batch (host arrays), or None. Recomputed only
        when the batch changes: shared pages are full prompt pages, which never change."""
        if not self._cascade_on:
            return None
        key = tuple(id(r) for r in reqs)
        if key == self._casc_key:
            return self._casc_plan
        from ..ops.attention import cascade_groups

        groups = cascade_groups([r.blocks for r in reqs], self.cfg.cascade_min_pages,
                                [len(r.prompt) // PAGE for r in reqs])
        plan = None
        if groups:
            B = len(reqs)
            q_index, cu, lens, first_rows = [], [0], [], []
            row_of, page_start = [-1] * B, [0] * B
            for rows, shared in groups:
                for i in rows:
                    row_of[i] = len(q_index)
                    page_start[i] = shared
                    q_index.append(i)
                cu.append(len(q_index))
                lens.append(shared * PAGE)
                first_rows.append(reqs[rows[0]].row)
            plan = {"q_index": q_index, "cu_q": cu, "seq_lens": lens, "bt_rows": first_rows, "row_of": row_of,
                    "page_start": page_start, "max_q": max(len(g[0]) for g in groups),
                    "grouped": len(q_index), "serial": next(self._casc_serial)}
        self._casc_key, self._casc_plan = key, plan
        return plan

    def _cascade_meta_eager(self, plan: Optional[dict], max_seq_len: int):
        if plan is None:
            return None
        from ..ops.attention import CascadeMeta, cascade_num_splits

        q_index, cu, lens, row_of, ps = self._stage_int32(plan["q_index"], plan["cu_q"], plan["seq_lens"],
                                                         plan["row_of"], plan["page_start"])
        rows = torch.tensor(plan["bt_rows"], dtype=torch.long, device=self.device)
        ng = len(plan["seq_lens"])
        return CascadeMeta(q_index, cu, lens, self.block_table.index_select(0, rows), row_of, ps, plan["max_q"],
                           cascade_num_splits(ng, self.cache.num_kv_heads, max_seq_len, self.device))

    def _decode(self, reqs: List[Request]) -> List[Request]:
        if self.spec is not None and all(r.params.temperature <= 0 for r in reqs):
            return self.spec.step(reqs)
        toks, pos, slots, lens = self.decode_meta(reqs)
        self.stat["decode_tokens"] += len(reqs)
        plan = self.cascade_plan(reqs)
        if plan is not None:
            self.stat["cascade_steps"] += 1
            self.stat["cascade_grouped_seqs"] += plan["grouped"]
        if self._graphs is not None:
            logits = self._graphs.run(reqs, toks, pos, slots, lens, plan)[0]
        else:
            casc = self._cascade_meta_eager(plan, max(lens))
            d_toks, d_pos, d_slots, d_lens, d_rows = self._stage_int32(toks, pos, slots, lens, [r.row for r in reqs])
            meta = AttnMeta(mode="decode", positions=d_pos, slots=d_slots,
                            block_table=self.block_table.index_select(0, d_rows.long()), seq_lens=d_lens,
                            max_seq_len=max(lens), cascade=casc)
            logits = self.model.forward(d_toks, meta, self.cache)
        new = self._sample(logits, reqs)
        done: List[Request] = []
        for r, t in zip(reqs, new):
            self._append(r, t, done)
        return done

    # ------------------------------------------------------------------ telemetry
    def stats(self) -> Dict:
        out = dict(self.stat)
        out["blocks"] = self.bm.stats()
        if self.amf is not None:
            out["amf"] = self.amf.stats()
        if self.spec is not None:
            out["spec"] = self.spec.stats()
        return out
