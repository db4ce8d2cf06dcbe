"""Local reasoning model with LoRA adapters, and its DPO learning loop.

:class:`LocalReasoningModel` makes the policy decision with a language model held by this
process (any :class:`~..models.llama.LlamaModel`: a Hugging Face checkpoint through
``models/loader.py``, or random-init weights in tests). The state vector becomes a prompt
(slot name = value), and instead of parsing free text the model *ranks* a fixed set of
candidate decisions, each rendered as a compact JSON object: the candidate with the highest
log-likelihood given the prompt wins. Every answer is therefore a valid decision, and the
same score is what the learning loop trains.

:class:`LoRA` adds rank-``r`` adapters ``scale * B A`` to the attention and MLP projections
of every layer. :func:`lm_forward` is a differentiable PyTorch forward of the same model
(the serving kernels have no backward) that applies the adapters; :func:`dpo_step` trains
only the adapter parameters with Direct Preference Optimisation (Rafailov et al. 2023)
against the frozen base model as the reference policy, on pairs (state, preferred decision,
rejected decision) -- e.g. from the reward ledger. :meth:`LoRA.merge` folds the adapters
into the weights so the fused GPU kernels serve the fine-tuned model; :meth:`LoRA.unmerge`
restores them.

Reference counterparts: the local 8B NF4 reasoning model emitting decision vectors
(platform/reasoning/reasoning_model.py:183-326) and its LoRA PPO/DPO learning loop
(platform/reasoning/learning_loop.py:159).
"""
from __future__ import annotations

import json
import math
import os
import threading
import time
from dataclasses import dataclass
from itertools import product
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn.functional as F

from ..ops.dense import SWIGLU_GROUP
from .decide import DEPTHS, Decision
from .state import Slot

TARGETS = ("wqkv", "wo", "w_gate_up", "w_down")


class LoRA(torch.nn.Module):
    """Rank-``r`` adapters on the projections ``TARGETS`` of every layer of ``model``."""

    def __init__(self, model, r: int = 8, alpha: float = 16.0, seed: int = 0):
        super().__init__()
        self.model, self.r, self.scale = model, r, alpha / r
        g = torch.Generator().manual_seed(seed)
        self.A = torch.nn.ParameterDict()
        self.B = torch.nn.ParameterDict()
        for li, lw in enumerate(model.layers):
            for name in TARGETS:
                w = getattr(lw, name, None)
                if w is None:
                    continue
                out_f, in_f = w.shape
                key = f"{li}_{name}"
                # A random, B zero: the adapted model starts equal to the base model
                self.A[key] = torch.nn.Parameter(torch.randn(r, in_f, generator=g) / math.sqrt(in_f))
                self.B[key] = torch.nn.Parameter(torch.zeros(out_f, r))
        self.to(model.embed.device)
        self.merged = False

    def clone(self) -> "LoRA":
        """A trainable copy with the same keys, ranks and scaling (the model is shared)."""
        c = LoRA(self.model, self.r, self.scale * self.r)
        for key in list(c.A.keys()):
            if key not in self.A:
                del c.A[key], c.B[key]
        for key in self.A.keys():
            c.A[key] = torch.nn.Parameter(self.A[key].detach().clone())
            c.B[key] = torch.nn.Parameter(self.B[key].detach().clone())
        return c

    def delta(self, li: int, name: str) -> Optional[torch.Tensor]:
        key = f"{li}_{name}"
        if key not in self.A:
            return None
        return self.scale * (self.B[key] @ self.A[key])

    def merge(self) -> None:
        """W += scale B A for every adapted projection (serving with the fused kernels)."""
        if self.merged:
            return
        with torch.no_grad():
            for li, lw in enumerate(self.model.layers):
                for name in TARGETS:
                    d = self.delta(li, name)
                    if d is not None:
                        w = getattr(lw, name)
                        w.copy_((w.float() + d.to(w.device)).to(w.dtype))
        self.merged = True

    def unmerge(self) -> None:
        if not self.merged:
            return
        with torch.no_grad():
            for li, lw in enumerate(self.model.layers):
                for name in TARGETS:
                    d = self.delta(li, name)
                    if d is not None:
                        w = getattr(lw, name)
                        w.copy_((w.float() - d.to(w.device)).to(w.dtype))
        self.merged = False


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def lm_forward(model, tokens: torch.Tensor, lora: Optional[LoRA] = None, start: int = 0,
               past: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None, return_kv: bool = False):
    """Differentiable causal forward of a dense ``LlamaModel`` over ``tokens`` [B, T] (or
    [T]) -> logits [B, T, vocab] (or [T, vocab]) in fp32, with ``lora``'s adapters applied
    unless they are merged. Rows are independent; right padding does not change the logits
    of the positions before it. Matmuls run in fp32 on the CPU and in the weights' dtype on
    the GPU (fp32 accumulation).

    ``past`` (per layer (K, V) [1, P, Hq, D] of a shared prefix, from a call with
    ``return_kv=True``) continues every row after that prefix: positions start at ``start``
    (= P) and each row attends to the whole prefix, then causally to itself. With
    ``return_kv`` the result is (logits, per-layer (K, V) of this call's tokens)."""
    cfg = model.cfg
    squeeze = tokens.dim() == 1
    if squeeze:
        tokens = tokens[None]
    B, T = tokens.shape
    Hq, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    cd = torch.float32 if tokens.device.type == "cpu" else model.dtype
    pos = torch.arange(start, start + T, device=tokens.device)
    cs = model.cos_sin.to(tokens.device)[pos].float()
    half = D // 2
    cos, sin = cs[None, :, None, :half], cs[None, :, None, half:]
    use = lora is not None and not lora.merged
    P = past[0][0].shape[1] if past else 0
    mask = None
    if P:  # prefix fully visible, own tokens causal
        own = torch.ones(T, T, dtype=torch.bool, device=tokens.device).tril()
        mask = torch.cat((torch.ones(T, P, dtype=torch.bool, device=tokens.device), own), dim=1)

    def proj(x, li, name, w):
        y = (x.to(cd) @ w.to(cd).t()).float()
        if use:
            d = lora.delta(li, name)
            if d is not None:
                y = y + x @ d.to(x.device).t()
        return y

    def rope(x):
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat((x1 * cos - x2 * sin, x2 * cos + x1 * sin), dim=-1)

    h = model.embed[tokens.long()].float()
    rep = Hq // Hkv
    kv_out = []
    for li, lw in enumerate(model.layers):
        if lw.w_gate_up is None:
            raise ValueError("lm_forward: dense (non-MoE) models only")
        x = _rms(h, lw.attn_norm, cfg.rms_eps)
        qkv = proj(x, li, "wqkv", lw.wqkv).view(B, T, Hq + 2 * Hkv, D)
        q = rope(qkv[:, :, :Hq])
        k = rope(qkv[:, :, Hq:Hq + Hkv]).repeat_interleave(rep, dim=2)
        v = qkv[:, :, Hq + Hkv:].repeat_interleave(rep, dim=2)
        if return_kv:
            kv_out.append((k, v))
        if P:
            k = torch.cat((past[li][0].expand(B, -1, -1, -1), k), dim=1)
            v = torch.cat((past[li][1].expand(B, -1, -1, -1), v), dim=1)
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               attn_mask=mask).transpose(1, 2)
        else:
            a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True).transpose(1, 2)
        h = h + proj(a.reshape(B, T, Hq * D), li, "wo", lw.wo)
        x = _rms(h, lw.mlp_norm, cfg.rms_eps)
        gu = proj(x, li, "w_gate_up", lw.w_gate_up)
        n = gu.shape[-1]
        g4 = gu.view(B, T, n // (2 * SWIGLU_GROUP), 2, SWIGLU_GROUP)  # gate/up interleaved by 64 rows
        act = (F.silu(g4[..., 0, :]) * g4[..., 1, :]).reshape(B, T, n // 2)
        h = h + proj(act, li, "w_down", lw.w_down)
    logits = (_rms(h, model.final_norm, cfg.rms_eps).to(cd) @ model.lm_head.to(cd).t()).float()
    logits = logits[0] if squeeze else logits
    return (logits, kv_out) if return_kv else logits


def candidate_decisions() -> List[Decision]:
    """The discrete decision set the model ranks: admission x speculative depth x back-pressure."""
    out = []
    for admit, depth, thr in product((True, False), DEPTHS, (0.0, 0.25, 0.5)):
        out.append(Decision(cache_admission=admit, spec_decode_depth=depth, spec_decode_enable=depth > 2,
                            throttle_back_pressure=thr))
    return out


def render(d: Decision) -> str:
    return json.dumps({"cache_admission": d.cache_admission, "spec_decode_depth": d.spec_decode_depth,
                       "throttle_back_pressure": d.throttle_back_pressure}, separators=(",", ":"))


class LocalReasoningModel:
    """Policy decisions from a local language model by ranking candidate decisions."""

    def __init__(self, model, tokenizer=None, lora: Optional[LoRA] = None,
                 candidates: Optional[Sequence[Decision]] = None, max_prompt_tokens: int = 256):
        self.model, self.tok, self.lora = model, tokenizer, lora
        self.candidates = list(candidates or candidate_decisions())
        self.max_prompt_tokens = max_prompt_tokens

    def encode(self, text: str) -> List[int]:
        if self.tok is not None:
            return list(self.tok.encode(text))
        return [b % self.model.cfg.vocab for b in text.encode()]  # bytes as token ids

    def prompt(self, v: np.ndarray) -> List[int]:
        """``state {slot: value, ...} decision `` over the non-zero named slots (in slot
        order), cut to ``max_prompt_tokens`` from the front so the early slots stay."""
        named = {k: round(float(v[i]), 3) for k, i in sorted(((k, i) for k, i in vars(Slot).items()
                                                              if k.isupper() and isinstance(i, int)), key=lambda x: x[1])
                 if i < len(v) and abs(float(v[i])) >= 5e-4}
        body = self.encode("state " + json.dumps(named, separators=(",", ":")))
        return body[:self.max_prompt_tokens] + self.encode(" decision ")

    def scores(self, v: np.ndarray, lora: Optional[LoRA] = None,
               candidates: Optional[Sequence[Decision]] = None) -> torch.Tensor:
        """Log-likelihood of every candidate given the state prompt [len(candidates)]: the
        prompt runs once, and all candidates (right-padded rows) continue from its K/V."""
        p = self.prompt(v)
        cands = [self.encode(render(d)) for d in (candidates if candidates is not None else self.candidates)]
        dev = self.model.embed.device
        plog, kv = lm_forward(self.model, torch.tensor([p], dtype=torch.long, device=dev), lora, return_kv=True)
        first = F.log_softmax(plog[0, -1], dim=-1)  # the prompt's last position predicts token 0
        T = max(len(c) for c in cands)
        toks = torch.tensor([c + [0] * (T - len(c)) for c in cands], dtype=torch.long, device=dev)
        out = first[toks[:, 0]]
        if T > 1:
            lp = F.log_softmax(lm_forward(self.model, toks[:, :-1], lora, start=len(p), past=kv), dim=-1)
            tok_lp = lp.gather(2, toks[:, 1:, None])[..., 0]
            mask = torch.zeros(len(cands), T - 1, device=dev)
            for i, c in enumerate(cands):
                mask[i, :len(c) - 1] = 1.0
            out = out + (tok_lp * mask).sum(1)
        return out

    def policy_logprob(self, v: np.ndarray, d: Decision, lora: Optional[LoRA] = None) -> torch.Tensor:
        """log pi(d | state) of the policy that picks among the candidates with probabilities
        softmax(scores); ``d`` joins the candidate set if it is not in it."""
        cands = list(self.candidates)
        idx = next((i for i, c in enumerate(cands) if render(c) == render(d)), None)
        if idx is None:
            cands.append(d)
            idx = len(cands) - 1
        return F.log_softmax(self.scores(v, lora, cands), dim=0)[idx]

    def decode_text(self, ids: List[int]) -> str:
        if self.tok is not None:
            return self.tok.decode(ids)
        return bytes(int(t) % 256 for t in ids).decode("utf-8", errors="replace")

    def generate(self, v: np.ndarray, max_new: int = 192, lora: Optional[LoRA] = None) -> Tuple[str, List[int]]:
        """Greedy free-form answer to the state prompt, one token at a time over the cached
        K/V of the prompt and the tokens so far; stops when the JSON object it opened closes."""
        dev = self.model.embed.device
        ids = self.prompt(v) + self.encode("{")
        logits, kv = lm_forward(self.model, torch.tensor([ids], dtype=torch.long, device=dev), lora, return_kv=True)
        out = list(self.encode("{"))
        depth, n = 1, len(ids)
        for _ in range(max_new):
            nxt = int(torch.argmax(logits[0, -1]))
            out.append(nxt)
            text = self.decode_text(out)
            depth = text.count("{") - text.count("}")
            if depth <= 0:
                break
            logits, new_kv = lm_forward(self.model, torch.tensor([[nxt]], dtype=torch.long, device=dev), lora,
                                        start=n, past=kv, return_kv=True)
            kv = [(torch.cat((pk, k), dim=1), torch.cat((pv, vv), dim=1)) for (pk, pv), (k, vv) in zip(kv, new_kv)]
            n += 1
        return self.decode_text(out), out

    def decide_generated(self, v: np.ndarray, max_new: int = 192) -> Decision:
        """The reference's way: the model writes the decision JSON itself (nested or flat
        fields); anything that does not parse or validate returns a fallback decision."""
        t0 = time.perf_counter()
        try:
            with torch.no_grad():
                text, _ = self.generate(v, max_new, self.lora)
            d = Decision.from_dict(json.loads(text[text.index("{"):text.rindex("}") + 1]))
            if d.validate():
                raise ValueError("; ".join(d.validate()))
        except Exception:
            d = Decision(is_fallback=True)
        d.inference_ms = (time.perf_counter() - t0) * 1e3
        return d

    def decide(self, v: np.ndarray) -> Decision:
        """The highest-scoring candidate; any failure returns a fallback decision (fail closed,
        like the endpoint model)."""
        t0 = time.perf_counter()
        try:
            with torch.no_grad():
                s = self.scores(v, self.lora)
            d = Decision(**self.candidates[int(torch.argmax(s))].to_dict())
        except Exception:
            d = Decision(is_fallback=True)
        d.inference_ms = (time.perf_counter() - t0) * 1e3
        return d


def dpo_step(lm: LocalReasoningModel, lora: LoRA, opt: torch.optim.Optimizer,
             pairs: Sequence[Tuple[np.ndarray, Decision, Decision]], beta: float = 0.1) -> float:
    """One DPO update of the adapters on (state, preferred, rejected) pairs; the reference
    policy is the base model (adapters off). Returns the mean loss."""
    losses = []
    for v, good, bad in pairs:
        with torch.no_grad():
            ref = lm.scores(v, None, [good, bad])
        cur = lm.scores(v, lora, [good, bad])
        margin = beta * ((cur[0] - ref[0]) - (cur[1] - ref[1]))
        losses.append(-F.logsigmoid(margin))
    loss = torch.stack(losses).mean()
    opt.zero_grad()
    loss.backward()
    opt.step()
    return float(loss.detach())


def preference_pairs(ledger_rows: Sequence[Dict]) -> List[Tuple]:
    """Pairs for :func:`dpo_step` from rows {state, decision, reward}: within groups of rows
    with the same rounded state, the highest-reward decision is preferred over the lowest."""
    groups: Dict[bytes, List[Dict]] = {}
    for r in ledger_rows:
        key = np.round(np.asarray(r["state"], dtype=np.float32), 2).tobytes()
        groups.setdefault(key, []).append(r)
    pairs = []
    for rows in groups.values():
        if len(rows) < 2:
            continue
        rows = sorted(rows, key=lambda r: r["reward"])
        lo, hi = rows[0], rows[-1]
        if hi["reward"] > lo["reward"]:
            pairs.append((np.asarray(hi["state"], dtype=np.float32), hi["decision"], lo["decision"]))
    return pairs


def sft_step(lm: LocalReasoningModel, lora: LoRA, opt: torch.optim.Optimizer,
             rows: Sequence[Tuple[np.ndarray, Decision, float]]) -> float:
    """One update raising the log-likelihood of each (state, decision) weighted by its
    ``weight``: weights 1 on positive-reward rows is supervised fine-tuning on good
    decisions; centred rewards as weights is REINFORCE with a mean baseline."""
    losses = [-w * lm.scores(v, lora, [d])[0] for v, d, w in rows]
    loss = torch.stack(losses).mean()
    opt.zero_grad()
    loss.backward()
    opt.step()
    return float(loss.detach())


def ppo_step(lm: LocalReasoningModel, lora: LoRA, opt: torch.optim.Optimizer,
             rows: Sequence[Tuple[np.ndarray, Decision, float, float]], clip: float = 0.2) -> float:
    """One clipped-surrogate PPO update (Schulman et al. 2017) on (state, decision,
    advantage, behaviour log-prob) rows; the policy is the softmax over the candidates'
    scores."""
    losses = []
    for v, d, adv, old_lp in rows:
        ratio = torch.exp(lm.policy_logprob(v, d, lora) - old_lp)
        losses.append(-torch.min(ratio * adv, torch.clamp(ratio, 1 - clip, 1 + clip) * adv))
    loss = torch.stack(losses).mean()
    opt.zero_grad()
    loss.backward()
    opt.step()
    return float(loss.detach())


@dataclass
class TrainingResult:
    examples_used: int
    mean_reward: float
    loss: float
    adapter_path: Optional[str]
    elapsed_s: float
    skipped: bool
    skip_reason: str = ""


class LoraLearningLoop:
    """Periodic LoRA fine-tuning of a :class:`LocalReasoningModel` from its own scored
    decisions in a :class:`~.learn.RewardLedger`. ``level`` picks the objective: 1 SFT on
    positive-reward decisions, 2 reward-weighted policy gradient (REINFORCE with a mean
    baseline), 3 PPO (clipped ratio, :func:`ppo_step`) over the model's distribution on the
    candidate decisions, 4 DPO on best-versus-worst pairs of the same state.
    Each cycle trains a copy of the live adapters and swaps it in under a lock, so
    ``decide`` never sees half-updated weights; the adapters are saved to ``adapter_dir``.
    """

    def __init__(self, lm: LocalReasoningModel, ledger, level: int = 4, interval_s: float = 3600.0,
                 batch_size: int = 64, min_examples: int = 8, epochs: int = 2, lr: float = 1e-3, beta: float = 0.1,
                 r: int = 8, alpha: float = 16.0, adapter_dir: Optional[str] = None, adapter_format: str = "peft"):
        self.lm, self.ledger, self.level = lm, ledger, int(level)
        self.interval_s, self.batch_size, self.min_examples = max(1.0, float(interval_s)), batch_size, min_examples
        self.epochs, self.lr, self.beta, self.r, self.alpha = epochs, lr, beta, r, alpha
        self.adapter_dir = adapter_dir
        if adapter_format not in ("peft", "pt"):
            raise ValueError("adapter_format must be 'peft' or 'pt'")
        self.adapter_format = adapter_format
        self.cycles = 0
        self._swap = threading.Lock()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    def _examples(self, rows) -> Tuple[str, list]:
        if self.level >= 4:
            return "dpo", preference_pairs(rows)
        if self.level == 3:
            mean = float(np.mean([r["reward"] for r in rows])) if rows else 0.0
            ex = [(r["state"], r["decision"], r["reward"] - mean) for r in rows if r["reward"] != mean]
            with torch.no_grad():  # behaviour policy: the live adapters before this cycle
                return "ppo", [(v, d, a, float(self.lm.policy_logprob(v, d, self.lm.lora))) for v, d, a in ex]
        if self.level >= 2:
            mean = float(np.mean([r["reward"] for r in rows])) if rows else 0.0
            return "pg", [(r["state"], r["decision"], r["reward"] - mean) for r in rows if r["reward"] != mean]
        return "sft", [(r["state"], r["decision"], 1.0) for r in rows if r["reward"] > 0]

    def run_once(self) -> TrainingResult:
        t0 = time.perf_counter()
        rows = self.ledger.scored(self.batch_size, consume=False)
        if not rows:
            return TrainingResult(0, 0.0, 0.0, None, time.perf_counter() - t0, True, "no scored decisions")
        kind, ex = self._examples(rows)
        if len(ex) < self.min_examples:
            return TrainingResult(len(ex), 0.0, 0.0, None, time.perf_counter() - t0, True,
                                  f"only {len(ex)} {kind} examples < {self.min_examples}")
        live = self.lm.lora
        if live is not None and live.merged:  # the weights carry its delta: training on them would count it twice
            return TrainingResult(len(ex), 0.0, 0.0, None, time.perf_counter() - t0, True,
                                  "live adapters are merged into the weights: unmerge before training")
        lora = live.clone() if live is not None else LoRA(self.lm.model, self.r, self.alpha)
        opt = torch.optim.AdamW(lora.parameters(), lr=self.lr)
        loss = 0.0
        try:
            for _ in range(self.epochs):
                if kind == "dpo":
                    loss = dpo_step(self.lm, lora, opt, ex, self.beta)
                elif kind == "ppo":
                    loss = ppo_step(self.lm, lora, opt, ex)
                else:
                    loss = sft_step(self.lm, lora, opt, ex)
        except Exception as e:  # the live adapters stay; the rows stay unconsumed for the next cycle
            return TrainingResult(len(ex), 0.0, 0.0, None, time.perf_counter() - t0, True, f"fine-tune error: {e}")
        with self._swap:
            self.lm.lora = lora
        self.ledger.scored(len(rows), consume=True)
        path = self.save(lora) if self.adapter_dir else None
        self.cycles += 1
        return TrainingResult(len(ex), float(np.mean([r["reward"] for r in rows])), loss, path,
                              time.perf_counter() - t0, False)

    def decide(self, v: np.ndarray) -> Decision:
        with self._swap:
            return self.lm.decide(v)

    def save(self, lora: LoRA) -> str:
        """This cycle's adapters under ``adapter_dir``: a PEFT adapter directory
        (``adapter_format="peft"``, loads with :func:`load_peft_adapter` or Hugging Face PEFT)
        or one ``.pt`` file (``"pt"``, :func:`load_adapter`)."""
        os.makedirs(self.adapter_dir, exist_ok=True)
        if self.adapter_format == "peft":
            path = os.path.join(self.adapter_dir, f"adapter_{self.cycles:05d}")
            save_peft_adapter(lora, path)
            return path
        path = os.path.join(self.adapter_dir, f"adapter_{self.cycles:05d}.pt")
        torch.save({"r": lora.r, "scale": lora.scale, "state": lora.state_dict()}, path)
        return path

    def start(self) -> None:
        if self._thread is not None and self._thread.is_alive():
            return
        self._stop.clear()
        self._thread = threading.Thread(target=self._run, daemon=True, name="lora-learning-loop")
        self._thread.start()

    def _run(self) -> None:
        while not self._stop.wait(self.interval_s):
            self.run_once()

    def stop(self, timeout: float = 10.0) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None


def load_adapter(model, path: str) -> LoRA:
    """A :class:`LoRA` for ``model`` with the weights saved by :meth:`LoraLearningLoop.save`."""
    blob = torch.load(path, map_location="cpu")
    lora = LoRA(model, blob["r"], blob["scale"] * blob["r"])
    lora.load_state_dict(blob["state"])
    return lora


# ------------------------------------------------------------------ PEFT adapter format
_PEFT_PREFIX = "base_model.model.model.layers.{}."
_PEFT_MODULES = {"wqkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "wo": ("self_attn.o_proj",),
                 "w_gate_up": ("mlp.gate_proj", "mlp.up_proj"), "w_down": ("mlp.down_proj",)}


def _gate_up_rows(F2: int, part: int) -> torch.Tensor:
    """Rows of the 64-row-interleaved gate/up matrix [2F, H] that belong to gate (part 0)
    or up (part 1), in order."""
    g = torch.arange(F2).view(F2 // (2 * SWIGLU_GROUP), 2, SWIGLU_GROUP)
    return g[:, part].reshape(-1)


def save_peft_adapter(lora: LoRA, path: str) -> None:
    """Writes ``lora`` as a Hugging Face PEFT adapter directory (``adapter_config.json`` +
    ``adapter_model.safetensors``; separate q/k/v and gate/up projections, which share the
    fused adapter's A and take their rows of its B)."""
    from ..models.loader import save_safetensors

    os.makedirs(path, exist_ok=True)
    cfg = lora.model.cfg
    q, kv = cfg.q_size, cfg.kv_size
    out: Dict[str, torch.Tensor] = {}
    rank_pattern: Dict[str, int] = {}
    alpha_pattern: Dict[str, float] = {}
    for li in range(len(lora.model.layers)):
        pre = _PEFT_PREFIX.format(li)
        for name, mods in _PEFT_MODULES.items():
            key = f"{li}_{name}"
            if key not in lora.A:
                continue
            A, B = lora.A[key].detach().float().cpu(), lora.B[key].detach().float().cpu()
            if A.shape[0] != lora.r:  # an imported fused adapter: its own rank, same scaling
                for mod in mods:
                    rank_pattern[f"model.layers.{li}.{mod}"] = int(A.shape[0])
                    alpha_pattern[f"model.layers.{li}.{mod}"] = lora.scale * A.shape[0]
            if name == "wqkv":
                parts = [B[:q], B[q:q + kv], B[q + kv:]]
            elif name == "w_gate_up":
                parts = [B[_gate_up_rows(B.shape[0], 0)], B[_gate_up_rows(B.shape[0], 1)]]
            else:
                parts = [B]
            for mod, b in zip(mods, parts):
                out[pre + mod + ".lora_A.weight"] = A.contiguous()
                out[pre + mod + ".lora_B.weight"] = b.contiguous()
    save_safetensors(os.path.join(path, "adapter_model.safetensors"), out)
    with open(os.path.join(path, "adapter_config.json"), "w") as f:
        json.dump({"peft_type": "LORA", "r": lora.r, "lora_alpha": lora.scale * lora.r,
                   "rank_pattern": rank_pattern, "alpha_pattern": alpha_pattern,
                   "target_modules": ["q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"],
                   "bias": "none", "task_type": "CAUSAL_LM"}, f, indent=1)


def load_peft_adapter(model, path: str) -> LoRA:
    """A :class:`LoRA` for ``model`` from a Hugging Face PEFT adapter directory. Separate
    q/k/v (gate/up) adapters become one adapter of the fused projection: A stacked, B block
    diagonal (its gate/up rows interleaved by 64 like the weights), so its delta is exactly
    the separate deltas stacked; projections the adapter does not cover get none."""
    from ..models.loader import SafetensorsFile

    with open(os.path.join(path, "adapter_config.json")) as f:
        conf = json.load(f)
    r, alpha = int(conf["r"]), float(conf.get("lora_alpha", conf["r"]))
    rank_pat, alpha_pat = conf.get("rank_pattern") or {}, conf.get("alpha_pattern") or {}

    def module_scale(module: str) -> float:
        """PEFT's alpha / r of this module (patterns match by suffix) over the global one."""
        r_m = next((int(v) for k, v in rank_pat.items() if module.endswith(k)), r)
        a_m = next((float(v) for k, v in alpha_pat.items() if module.endswith(k)), alpha)
        return (a_m / r_m) / (alpha / r)

    st = SafetensorsFile(os.path.join(path, "adapter_model.safetensors"))
    try:
        names = set(st.keys())
        cfg = model.cfg
        lora = LoRA(model, r, alpha)
        dev = model.embed.device
        for li, lw in enumerate(model.layers):
            pre = _PEFT_PREFIX.format(li)
            for name, mods in _PEFT_MODULES.items():
                key = f"{li}_{name}"
                w = getattr(lw, name, None)
                if w is None or key not in lora.A:
                    continue
                if name == "wqkv":
                    rows = [cfg.q_size, cfg.kv_size, cfg.kv_size]
                elif name == "w_gate_up":
                    rows = [w.shape[0] // 2, w.shape[0] // 2]
                else:
                    rows = [w.shape[0]]
                As, blocks = [], []  # blocks: (row offset in the [part0; part1; ...] layout, B block)
                off = 0
                for mod, nrow in zip(mods, rows):
                    a_n, b_n = pre + mod + ".lora_A.weight", pre + mod + ".lora_B.weight"
                    if a_n in names and b_n in names:
                        A_p, B_p = st.get(a_n).float(), st.get(b_n).float()
                        if B_p.shape[0] != nrow or A_p.shape[1] != w.shape[1] or B_p.shape[1] != A_p.shape[0]:
                            raise ValueError(f"{mod} of layer {li}: adapter shapes {tuple(A_p.shape)} / "
                                             f"{tuple(B_p.shape)} do not fit the projection")
                        As.append(A_p)
                        blocks.append((off, B_p * module_scale(f"model.layers.{li}.{mod}")))
                    off += nrow
                if not As:  # this projection has no adapter
                    del lora.A[key], lora.B[key]
                    continue
                A = torch.cat(As, dim=0)
                B = torch.zeros(w.shape[0], A.shape[0])
                col = 0
                for row0, B_p in blocks:
                    B[row0:row0 + B_p.shape[0], col:col + B_p.shape[1]] = B_p
                    col += B_p.shape[1]
                if name == "w_gate_up":  # [gate; up] rows -> the weights' 64-row interleave
                    F2 = w.shape[0]
                    inter = torch.empty_like(B)
                    inter[_gate_up_rows(F2, 0)] = B[:F2 // 2]
                    inter[_gate_up_rows(F2, 1)] = B[F2 // 2:]
                    B = inter
                lora.A[key] = torch.nn.Parameter(A.to(dev))
                lora.B[key] = torch.nn.Parameter(B.to(dev))
    finally:
        st.close()
    return lora


def main(argv: Optional[Sequence[str]] = None) -> int:
    """One offline learning cycle over a reward ledger:

        python -m axropus_deploy_b200.policy.local_model --ledger rewards.sqlite \\
            --model-dir /models/llama-3.1-8b --level 4 --out adapters/ [--adapter adapters/adapter_00003]

    trains (starting from ``--adapter`` when given) on the ledger's unconsumed scored
    decisions, writes the new adapters under ``--out`` and prints one JSON line."""
    import argparse

    from .learn import RewardLedger

    ap = argparse.ArgumentParser(description="one LoRA learning cycle of the local reasoning model")
    ap.add_argument("--ledger", required=True)
    ap.add_argument("--model-dir", required=True)
    ap.add_argument("--out", required=True)
    ap.add_argument("--level", type=int, default=4)
    ap.add_argument("--adapter", default=None, help="PEFT adapter directory to continue from")
    ap.add_argument("--epochs", type=int, default=2)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--min-examples", type=int, default=8)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    from ..models.loader import load_pretrained
    from ..server.app import load_tokenizer

    model = load_pretrained(a.model_dir, a.device)
    lm = LocalReasoningModel(model, load_tokenizer(a.model_dir))
    if a.adapter:
        lm.lora = load_peft_adapter(model, a.adapter)
    loop = LoraLearningLoop(lm, RewardLedger(a.ledger), level=a.level, epochs=a.epochs, lr=a.lr,
                            min_examples=a.min_examples, adapter_dir=a.out)
    r = loop.run_once()
    print(json.dumps({k: getattr(r, k) for k in ("examples_used", "mean_reward", "loss", "adapter_path", "elapsed_s",
                                                 "skipped", "skip_reason")}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
