"""Local reasoning model with LoRA adapters: differentiable forward, candidate ranking,
merge/unmerge, DPO / SFT / policy-gradient updates and the learning loop (CPU, fp32)."""
import json

import numpy as np
import pytest
import torch

from axropus_deploy_b200.models.config import ModelConfig
from axropus_deploy_b200.models.llama import LlamaModel
from axropus_deploy_b200.policy.decide import Decision
from axropus_deploy_b200.policy.learn import RewardLedger
from axropus_deploy_b200.policy.local_model import (LoRA, LocalReasoningModel, LoraLearningLoop, dpo_step,
                                                    load_adapter, lm_forward, preference_pairs, sft_step)
from axropus_deploy_b200.policy.state import WIDTH

MICRO = ModelConfig("micro", 2, 64, 4, 2, 16, 128, 320, 10000.0, None, max_position=1024)


def _model(seed=0):
    return LlamaModel(MICRO, "cpu", dtype=torch.float32, seed=seed, init_std=0.1)


def _sdpa_free_forward(model, toks):
    """Token-by-token fp32 forward with explicit softmax attention (no SDPA, no batching)."""
    cfg = model.cfg
    T = toks.shape[0]
    Hq, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim

    def rms(x, w):
        return x / torch.sqrt((x * x).mean(-1, keepdim=True) + cfg.rms_eps) * w

    def rope(x, p):
        c, s = model.cos_sin[p, :D // 2], model.cos_sin[p, D // 2:]
        a, b = x[..., :D // 2], x[..., D // 2:]
        return torch.cat((a * c - b * s, b * c + a * s), -1)

    h = model.embed[toks]
    for lw in model.layers:
        x = rms(h, lw.attn_norm)
        qkv = (x @ lw.wqkv.t()).view(T, Hq + 2 * Hkv, D)
        out = torch.zeros(T, Hq, D)
        for t in range(T):
            for hq in range(Hq):
                hk = hq // (Hq // Hkv)
                q = rope(qkv[t, hq], t)
                ks = torch.stack([rope(qkv[j, Hq + hk], j) for j in range(t + 1)])
                vs = qkv[: t + 1, Hq + Hkv + hk]
                w = torch.softmax(ks @ q / D ** 0.5, 0)
                out[t, hq] = w @ vs
        h = h + out.reshape(T, -1) @ lw.wo.t()
        x = rms(h, lw.mlp_norm)
        gu = x @ lw.w_gate_up.t()
        g = gu.view(T, -1, 2, 64)
        h = h + (torch.nn.functional.silu(g[:, :, 0]) * g[:, :, 1]).reshape(T, -1) @ lw.w_down.t()
    return rms(h, model.final_norm) @ model.lm_head.t()


def test_lm_forward_matches_explicit_attention():
    m = _model()
    toks = torch.randint(0, MICRO.vocab, (9,), generator=torch.Generator().manual_seed(1))
    ref = _sdpa_free_forward(m, toks)
    out = lm_forward(m, toks)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    # batched with right padding: rows unchanged before the padding
    b = torch.stack([toks, torch.cat([toks[:5], torch.zeros(4, dtype=torch.long)])])
    outb = lm_forward(m, b)
    torch.testing.assert_close(outb[0], ref, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(outb[1, :5], ref[:5], rtol=1e-4, atol=1e-4)


def test_lora_zero_init_merge_unmerge():
    m = _model()
    lora = LoRA(m, r=4)
    toks = torch.arange(12) % MICRO.vocab
    base = lm_forward(m, toks)
    torch.testing.assert_close(lm_forward(m, toks, lora), base)  # B = 0: adapted == base
    with torch.no_grad():
        for p in lora.B.values():
            p.normal_(0, 0.05)
    adapted = lm_forward(m, toks, lora)
    assert (adapted - base).abs().max() > 1e-3
    w0 = m.layers[0].wqkv.clone()
    lora.merge()
    torch.testing.assert_close(lm_forward(m, toks), adapted, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(lm_forward(m, toks, lora), adapted, rtol=1e-4, atol=1e-4)  # merged: not applied twice
    lora.unmerge()
    torch.testing.assert_close(m.layers[0].wqkv, w0, rtol=0, atol=1e-6)
    torch.testing.assert_close(lm_forward(m, toks), base, rtol=1e-4, atol=1e-4)


def test_scores_are_candidate_log_likelihoods():
    m = _model()
    lm = LocalReasoningModel(m, max_prompt_tokens=48)
    v = np.random.default_rng(0).random(WIDTH).astype(np.float32)
    s = lm.scores(v)
    assert s.shape == (len(lm.candidates),) and torch.isfinite(s).all() and (s < 0).all()
    # one candidate alone scores the same as inside the padded batch
    d = lm.candidates[5]
    torch.testing.assert_close(lm.scores(v, candidates=[d])[0], s[5], rtol=1e-4, atol=1e-3)
    dec = lm.decide(v)
    assert dec.to_dict()["spec_decode_depth"] == lm.candidates[int(torch.argmax(s))].spec_decode_depth
    assert dec.inference_ms > 0 and not dec.validate()


def _pair(lm):
    v = np.linspace(0, 1, WIDTH, dtype=np.float32)
    s = lm.scores(v).detach()
    good = lm.candidates[int(torch.argmin(s))]  # the base model's least likely decision
    bad = lm.candidates[int(torch.argmax(s))]
    return v, good, bad


def test_dpo_moves_decision_to_preferred():
    torch.manual_seed(0)
    m = _model()
    lm = LocalReasoningModel(m, max_prompt_tokens=32)
    v, good, bad = _pair(lm)
    lora = LoRA(m, r=4, alpha=8)
    lm.lora = lora
    opt = torch.optim.Adam(lora.parameters(), lr=2e-2)
    losses = [dpo_step(lm, lora, opt, [(v, good, bad)], beta=0.5) for _ in range(25)]
    assert losses[-1] < losses[0] * 0.5
    with torch.no_grad():
        s = lm.scores(v, lora, [good, bad])
    assert s[0] > s[1]


def test_sft_raises_likelihood():
    m = _model()
    lm = LocalReasoningModel(m, max_prompt_tokens=32)
    v, good, _ = _pair(lm)
    lora = LoRA(m, r=4)
    opt = torch.optim.Adam(lora.parameters(), lr=1e-2)
    before = float(lm.scores(v, lora, [good])[0].detach())
    for _ in range(10):
        sft_step(lm, lora, opt, [(v, good, 1.0)])
    assert float(lm.scores(v, lora, [good])[0].detach()) > before + 1.0


def test_preference_pairs_group_by_state():
    a = np.zeros(WIDTH, np.float32)
    b = np.ones(WIDTH, np.float32)
    d1, d2, d3 = Decision(spec_decode_depth=2), Decision(spec_decode_depth=8), Decision(spec_decode_depth=16)
    rows = [{"state": a, "decision": d1, "reward": -1.0}, {"state": a + 1e-4, "decision": d2, "reward": 2.0},
            {"state": a, "decision": d3, "reward": 0.5}, {"state": b, "decision": d1, "reward": 1.0}]
    pairs = preference_pairs(rows)
    assert len(pairs) == 1
    _, good, bad = pairs[0]
    assert good.spec_decode_depth == 8 and bad.spec_decode_depth == 2


@pytest.mark.parametrize("level", [1, 2, 3, 4])
def test_learning_loop_cycle(tmp_path, level):
    m = _model()
    lm = LocalReasoningModel(m, max_prompt_tokens=24)
    led = RewardLedger()
    rng = np.random.default_rng(0)
    states = [rng.random(WIDTH).astype(np.float32) for _ in range(3)]
    for v in states:
        for d, outcome in ((Decision(spec_decode_depth=8), "spec_high_acceptance"),
                           (Decision(spec_decode_depth=2, cache_admission=False), "spec_low_acceptance")):
            led.record_outcome(led.record_decision(d, v), outcome)
    loop = LoraLearningLoop(lm, led, level=level, min_examples=3, epochs=2, lr=1e-2, r=4,
                            adapter_dir=str(tmp_path))
    res = loop.run_once()
    assert not res.skipped, res.skip_reason
    assert res.examples_used >= 3 and res.adapter_path and lm.lora is not None
    assert led.scored(100) == []  # consumed
    again = loop.run_once()
    assert again.skipped
    from axropus_deploy_b200.policy.local_model import load_peft_adapter

    back = load_peft_adapter(m, res.adapter_path)  # PEFT directory by default
    for k in lm.lora.A:
        li, name = k.split("_", 1)
        torch.testing.assert_close(back.delta(int(li), name), lm.lora.delta(int(li), name), rtol=1e-5, atol=1e-6)
    pt = LoraLearningLoop(lm, led, adapter_dir=str(tmp_path / "pt"), adapter_format="pt").save(lm.lora)
    back = load_adapter(m, pt)
    for k in back.A:
        torch.testing.assert_close(back.A[k], lm.lora.A[k])
        torch.testing.assert_close(back.B[k], lm.lora.B[k])
    assert isinstance(loop.decide(states[0]), Decision)


def test_learning_loop_skips_without_data():
    m = _model()
    loop = LoraLearningLoop(LocalReasoningModel(m), RewardLedger(), interval_s=1)
    r = loop.run_once()
    assert r.skipped and "no scored" in r.skip_reason
    loop.start()
    loop.stop()


def test_learning_loop_survives_training_error(monkeypatch):
    import axropus_deploy_b200.policy.local_model as lm_mod

    m = _model()
    lm = LocalReasoningModel(m, max_prompt_tokens=24)
    led = RewardLedger()
    v = np.zeros(WIDTH, np.float32)
    for d, o in ((Decision(spec_decode_depth=8), "spec_high_acceptance"), (Decision(spec_decode_depth=2), "spec_low_acceptance")):
        led.record_outcome(led.record_decision(d, v), o)
    loop = LoraLearningLoop(lm, led, level=4, min_examples=1)

    def boom(*a, **k):
        raise RuntimeError("out of memory")
    monkeypatch.setattr(lm_mod, "dpo_step", boom)
    r = loop.run_once()
    assert r.skipped and "fine-tune error" in r.skip_reason and lm.lora is None
    assert len(led.scored(10, consume=False)) == 2  # still there for the next cycle


def test_dpo_learns_a_state_conditional_choice():
    """Two states that differ in one slot want opposite decisions; DPO on both pairs makes
    the model's choice follow the slot (the prompt keeps that slot)."""
    from axropus_deploy_b200.policy.state import Slot

    m = _model()
    shallow, deep = Decision(spec_decode_depth=2), Decision(spec_decode_depth=8)
    lm = LocalReasoningModel(m, candidates=[shallow, deep], max_prompt_tokens=48)
    lo, hi = np.zeros(WIDTH, np.float32), np.zeros(WIDTH, np.float32)
    lo[Slot.HIT_RATE], hi[Slot.HIT_RATE] = 0.1, 0.9
    assert lm.prompt(lo) != lm.prompt(hi)
    lora = LoRA(m, r=4, alpha=8)
    lm.lora = lora
    opt = torch.optim.Adam(lora.parameters(), lr=2e-2)
    for _ in range(30):
        dpo_step(lm, lora, opt, [(hi, deep, shallow), (lo, shallow, deep)], beta=0.5)
    assert lm.decide(hi).spec_decode_depth == 8 and lm.decide(lo).spec_decode_depth == 2


def test_adaptive_policy_consults_the_local_model():
    from axropus_deploy_b200.policy import AdaptivePolicy

    m = _model()
    lm = LocalReasoningModel(m, candidates=[Decision(spec_decode_depth=12, cache_admission=False)], max_prompt_tokens=32)
    pol = AdaptivePolicy(model=lm, model_primary=True)
    d = pol.decide(np.zeros(WIDTH, np.float32), "t1", "abc")
    assert d.spec_decode_depth == 12 and d.cache_admission is False and pol.stat["model"] == 1

    class Broken(LocalReasoningModel):
        def scores(self, *a, **k):
            raise RuntimeError("device lost")

    pol2 = AdaptivePolicy(model=Broken(m), model_primary=True)
    d2 = pol2.decide(np.zeros(WIDTH, np.float32), "t1", "abc")  # falls back to the local rules
    assert pol2.stat["model_failures"] == 1 and pol2.stat["local"] == 1 and not d2.validate()


def test_fedavg_of_lora_deltas():
    """Two nodes tune copies of the same adapters on different pairs; the sample-weighted
    FedAvg of their deltas (the federated loop's payload) loads back into an adapter."""
    from axropus_deploy_b200.policy.learn import fedavg, state_delta

    m = _model()
    lm = LocalReasoningModel(m, candidates=[Decision(spec_decode_depth=2), Decision(spec_decode_depth=8)],
                             max_prompt_tokens=32)
    base = LoRA(m, r=4)
    base_state = {k: v.clone() for k, v in base.state_dict().items()}
    v = np.linspace(0, 1, WIDTH, dtype=np.float32)
    deltas = []
    for node, (good, bad), n in ((0, (1, 0), 3), (1, (0, 1), 1)):
        lora = LoRA(m, r=4)
        lora.load_state_dict(base_state)
        opt = torch.optim.Adam(lora.parameters(), lr=1e-2)
        for _ in range(3):
            dpo_step(lm, lora, opt, [(v, lm.candidates[good], lm.candidates[bad])])
        deltas.append((state_delta(lora, base_state), n))
    avg = fedavg(deltas)
    merged = LoRA(m, r=4)
    merged.load_state_dict({k: base_state[k] + torch.as_tensor(avg[k]) for k in base_state})
    for k, t in merged.state_dict().items():
        want = base_state[k] + (3 * torch.as_tensor(deltas[0][0][k]) + torch.as_tensor(deltas[1][0][k])) / 4
        torch.testing.assert_close(t, want, rtol=1e-5, atol=1e-6)
    assert any(float(np.abs(a).max()) > 0 for a in avg.values())


def test_shared_prompt_scores_match_full_sequences():
    """Scores from one prompt pass + candidates continuing from its K/V equal the
    log-likelihoods of the whole (prompt + candidate) sequences, adapters included."""
    import torch.nn.functional as F

    from axropus_deploy_b200.policy.local_model import render

    m = _model()
    lora = LoRA(m, r=4)
    with torch.no_grad():
        for p_ in lora.B.values():
            p_.normal_(0, 0.05)
    lm = LocalReasoningModel(m, max_prompt_tokens=40)
    v = np.random.default_rng(3).random(WIDTH).astype(np.float32)
    got = lm.scores(v, lora)
    p = lm.prompt(v)
    want = []
    for d in lm.candidates:
        c = lm.encode(render(d))
        toks = torch.tensor(p + c)
        lp = F.log_softmax(lm_forward(m, toks, lora)[len(p) - 1:-1], dim=-1)
        want.append(lp.gather(1, toks[len(p):, None]).sum())
    torch.testing.assert_close(got, torch.stack(want), rtol=1e-4, atol=2e-3)


def test_peft_adapter_import_export(tmp_path):
    """A PEFT-format adapter (separate q/k/v/o/gate/up/down, random A and B) loaded onto the
    fused projections gives the same forward as the base weights with each projection's
    delta added the plain way; exporting it again and re-importing keeps the deltas."""
    from axropus_deploy_b200.models.loader import save_safetensors
    from axropus_deploy_b200.ops.dense import interleave_gate_up, split_gate_up
    from axropus_deploy_b200.policy.local_model import load_peft_adapter, save_peft_adapter

    m = _model()
    cfg = m.cfg
    H, q, kv, F_ = cfg.hidden, cfg.q_size, cfg.kv_size, cfg.ffn
    g = torch.Generator().manual_seed(5)
    shapes = {"self_attn.q_proj": (q, H), "self_attn.k_proj": (kv, H), "self_attn.v_proj": (kv, H),
              "self_attn.o_proj": (H, q), "mlp.gate_proj": (F_, H), "mlp.up_proj": (F_, H), "mlp.down_proj": (H, F_)}
    r, alpha = 4, 8.0
    tensors, deltas = {}, {}
    for li in range(len(m.layers)):
        for mod, (o, i) in shapes.items():
            if li == 1 and mod == "self_attn.k_proj":
                continue  # an uncovered part
            A = torch.randn(r, i, generator=g) * 0.1
            B = torch.randn(o, r, generator=g) * 0.1
            tensors[f"base_model.model.model.layers.{li}.{mod}.lora_A.weight"] = A
            tensors[f"base_model.model.model.layers.{li}.{mod}.lora_B.weight"] = B
            deltas[(li, mod)] = (alpha / r) * B @ A
    d = tmp_path / "peft"
    d.mkdir()
    save_safetensors(str(d / "adapter_model.safetensors"), tensors)
    (d / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "r": r, "lora_alpha": alpha}))
    lora = load_peft_adapter(m, str(d))
    toks = torch.arange(20) * 7 % cfg.vocab
    got = lm_forward(m, toks, lora)

    ref = _model()  # same seed: same base weights
    z = lambda o, i: torch.zeros(o, i)  # noqa: E731
    for li, lw in enumerate(ref.layers):
        dq = deltas[(li, "self_attn.q_proj")]
        dk = deltas.get((li, "self_attn.k_proj"), z(kv, H))
        dv = deltas[(li, "self_attn.v_proj")]
        lw.wqkv += torch.cat([dq, dk, dv])
        lw.wo += deltas[(li, "self_attn.o_proj")]
        gate, up = split_gate_up(lw.w_gate_up)
        lw.w_gate_up.copy_(interleave_gate_up(gate + deltas[(li, "mlp.gate_proj")], up + deltas[(li, "mlp.up_proj")]))
        lw.w_down += deltas[(li, "mlp.down_proj")]
    torch.testing.assert_close(got, lm_forward(ref, toks), rtol=1e-4, atol=1e-4)

    save_peft_adapter(lora, str(tmp_path / "out"))
    back = load_peft_adapter(m, str(tmp_path / "out"))
    for key in lora.A:
        li, name = key.split("_", 1)
        torch.testing.assert_close(back.delta(int(li), name), lora.delta(int(li), name), rtol=1e-5, atol=1e-6)
    conf = json.loads((tmp_path / "out" / "adapter_config.json").read_text())
    assert conf["rank_pattern"]["model.layers.0.self_attn.q_proj"] == 3 * r  # fused q/k/v rank


def test_ppo_moves_probability_to_the_rewarded_decision():
    from axropus_deploy_b200.policy.local_model import ppo_step

    m = _model()
    lo_d, hi_d = Decision(spec_decode_depth=2), Decision(spec_decode_depth=8)
    lm = LocalReasoningModel(m, candidates=[lo_d, hi_d], max_prompt_tokens=32)
    v = np.linspace(0, 1, WIDTH, dtype=np.float32)
    lora = LoRA(m, r=4, alpha=8)
    p0 = float(torch.exp(lm.policy_logprob(v, hi_d, lora)).detach())
    opt = torch.optim.Adam(lora.parameters(), lr=1e-2)
    for _ in range(4):  # a few cycles: behaviour log-probs refreshed each time, 3 epochs each
        with torch.no_grad():
            rows = [(v, hi_d, 1.0, float(lm.policy_logprob(v, hi_d, lora))),
                    (v, lo_d, -1.0, float(lm.policy_logprob(v, lo_d, lora)))]
        for _ in range(3):
            ppo_step(lm, lora, opt, rows)
    p1 = float(torch.exp(lm.policy_logprob(v, hi_d, lora)).detach())
    assert p1 > p0 + 0.2 and p1 > 0.7


def test_orchestrator_with_local_model_and_lora_loop():
    """The worker hooks with the local model as the policy's model and its LoRA loop
    training on the orchestrator's own reward ledger."""
    from axropus_deploy_b200.cluster.runtime import SpecKController
    from axropus_deploy_b200.policy import AdaptivePolicy, DecisionExecutor, PolicyOrchestrator, StateCollector

    m = _model()
    lm = LocalReasoningModel(m, candidates=[Decision(spec_decode_depth=4), Decision(spec_decode_depth=8)],
                             max_prompt_tokens=32)
    led = RewardLedger()
    loop = LoraLearningLoop(lm, led, level=2, min_examples=1, epochs=1, r=4)
    orch = PolicyOrchestrator(StateCollector(), policy=AdaptivePolicy(model=loop, model_primary=True),
                              executor=DecisionExecutor(SpecKController(4)), rewards=led)
    for i, acc in enumerate((9, 1)):
        tok = orch.before_job({"org_id": "acme", "fingerprint_hash": f"fp{i}"})
        assert tok is not None and tok[1].spec_decode_depth in (4, 8)
        orch.after_job(tok, {"amf": {"decision": "hit", "tier": "g1_raw", "saved_ms": 50.0},
                             "spec": {"drafted": 10, "accepted": acc}, "perf": {}}, mode="speculative")
    assert orch.policy.stat["model"] == 2
    r = loop.run_once()
    assert not r.skipped and lm.lora is not None


def test_generate_reuses_the_cache_and_parses_decisions(monkeypatch):
    import axropus_deploy_b200.policy.local_model as lmm

    m = _model()
    lm = LocalReasoningModel(m, max_prompt_tokens=24)
    v = np.zeros(WIDTH, np.float32)
    text, ids = lm.generate(v, max_new=6)
    # the incremental logits pick the same tokens as full-sequence forwards
    full = lm.prompt(v) + ids
    n0 = len(lm.prompt(v)) + 1
    ref = lm_forward(m, torch.tensor(full[:-1]))
    assert [int(t) for t in ref[n0 - 1:].argmax(-1)] == ids[1:]

    want = '{"decode": {"spec_decode_depth": 12}, "cache_admission": false}'
    real = lmm.lm_forward

    def scripted(model, tokens, lora=None, start=0, past=None, return_kv=False):
        logits, kv = real(model, tokens, lora, start, past, return_kv=True)
        produced = start + tokens.shape[1] - len(lm.prompt(v))  # tokens of the answer so far
        forced = torch.full_like(logits, -1e9)
        forced[..., ord(want[produced]) if produced < len(want) else 0] = 0.0
        return (forced, kv) if return_kv else forced

    monkeypatch.setattr(lmm, "lm_forward", scripted)
    d = lm.decide_generated(v)
    assert not d.is_fallback and d.spec_decode_depth == 12 and d.cache_admission is False
    monkeypatch.setattr(lmm, "lm_forward", real)
    assert lm.decide_generated(v, max_new=4).is_fallback  # an unfinished answer falls back


def test_offline_learning_cycle_cli(tmp_path, capsys):
    """``python -m axropus_deploy_b200.policy.local_model``: a saved checkpoint and a ledger
    file in, a PEFT adapter directory out; a second cycle continues from it."""
    from axropus_deploy_b200.models.loader import save_pretrained
    from axropus_deploy_b200.policy.local_model import main

    m = _model()
    save_pretrained(m, str(tmp_path / "ckpt"))
    led = RewardLedger(str(tmp_path / "rewards.sqlite"))
    v = np.zeros(WIDTH, np.float32)
    for d, o in ((Decision(spec_decode_depth=8), "spec_high_acceptance"), (Decision(spec_decode_depth=2), "spec_low_acceptance")):
        led.record_outcome(led.record_decision(d, v), o)
    args = ["--ledger", str(tmp_path / "rewards.sqlite"), "--model-dir", str(tmp_path / "ckpt"), "--out",
            str(tmp_path / "ad"), "--level", "4", "--min-examples", "1", "--device", "cpu"]
    assert main(args) == 0
    out = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert not out["skipped"] and out["adapter_path"].endswith("adapter_00000")
    led.record_outcome(led.record_decision(Decision(spec_decode_depth=8), v), "spec_high_acceptance")
    led.record_outcome(led.record_decision(Decision(spec_decode_depth=2), v), "spec_low_acceptance")
    assert main(args + ["--adapter", out["adapter_path"]]) == 0
    out2 = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert not out2["skipped"]
