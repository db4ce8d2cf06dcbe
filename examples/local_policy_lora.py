"""A local reasoning model choosing decisions and learning from their rewards with LoRA.

The model (a Hugging Face Llama checkpoint given with ``--model-dir``, else a small
random-init model) ranks candidate decisions for synthetic node states; each decision's
outcome comes from a fixed rule (deep speculation pays off when the acceptance slot is high,
shallow when it is low) and goes into the reward ledger; the DPO learning loop then tunes
LoRA adapters on best-versus-worst decisions of the same state, and the agreement of the
model's choices with the rule is printed before and after. Runs on cuda:0 when present, else
on the CPU. Prints one JSON line.

    python examples/local_policy_lora.py [--model-dir DIR] [--cycles 3]
"""
import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
from axropus_deploy_b200.models.config import ModelConfig  # noqa: E402
from axropus_deploy_b200.models.llama import LlamaModel  # noqa: E402
from axropus_deploy_b200.policy import LocalReasoningModel, LoraLearningLoop, RewardLedger, Slot  # noqa: E402
from axropus_deploy_b200.policy.decide import Decision  # noqa: E402
from axropus_deploy_b200.policy.state import WIDTH  # noqa: E402

CANDIDATES = [Decision(spec_decode_depth=d, spec_decode_enable=d > 2) for d in (2, 8)]


def rule(v: np.ndarray) -> int:
    """Depth the outcome rewards: 8 when recent acceptance (hit rate slot) is high, else 2."""
    return 8 if v[Slot.HIT_RATE] > 0.5 else 2


def agreement(lm, states) -> float:
    return float(np.mean([lm.decide(v).spec_decode_depth == rule(v) for v in states]))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--model-dir", default=None)
    ap.add_argument("--cycles", type=int, default=3)
    ap.add_argument("--states", type=int, default=8)
    ap.add_argument("--epochs", type=int, default=10)
    a = ap.parse_args()
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    tok = None
    if a.model_dir:
        from axropus_deploy_b200.models.loader import load_pretrained
        from axropus_deploy_b200.server.app import load_tokenizer

        model = load_pretrained(a.model_dir, dev)
        tok = load_tokenizer(a.model_dir)
    else:
        cfg = ModelConfig("policy-small", 2, 128, 4, 2, 32, 256, 512, 10000.0, None, max_position=2048)
        model = LlamaModel(cfg, dev, dtype=torch.float32 if dev == "cpu" else torch.bfloat16, seed=0, init_std=0.05)
    lm = LocalReasoningModel(model, tok, candidates=CANDIDATES, max_prompt_tokens=48)
    states = []
    for i in range(a.states):
        v = np.zeros(WIDTH, np.float32)
        v[Slot.HIT_RATE] = 0.9 if i % 2 else 0.1
        states.append(v)
    ledger = RewardLedger()
    loop = LoraLearningLoop(lm, ledger, level=4, min_examples=2, epochs=a.epochs, lr=2e-2, beta=0.5)
    before = agreement(lm, states)
    cycles = []
    for _ in range(a.cycles):
        for v in states:  # try both decisions on every state, score each by the rule
            for d in CANDIDATES:
                did = ledger.record_decision(d, v)
                ledger.record_outcome(did, "spec_depth_optimal" if d.spec_decode_depth == rule(v)
                                      else "spec_depth_wasteful")
        r = loop.run_once()
        cycles.append({"examples": r.examples_used, "loss": round(r.loss, 4), "skipped": r.skipped})
    print(json.dumps({"device": dev, "agreement_before": before, "agreement_after": agreement(lm, states),
                      "cycles": cycles}))


if __name__ == "__main__":
    main()
