"""The local reasoning model's differentiable forward against the serving kernels, and a
LoRA merged into the weights served by them (B200)."""
import numpy as np
import pytest
import torch


def _fused_logits(m, tokens):
    from axropus_deploy_b200.models.llama import AttnMeta
    from axropus_deploy_b200.ops.kvcache import KVCache

    cfg = m.cfg
    dev = tokens.device
    T = tokens.shape[0]
    pos = torch.arange(T, dtype=torch.int32, device=dev)
    bt = torch.arange(16, dtype=torch.int32, device=dev)[None]
    cache = KVCache(m.num_layers, 16, cfg.num_kv_heads, cfg.head_dim, "bf16", dev)
    meta = AttnMeta("prefill", pos, pos, bt, torch.tensor([T], dtype=torch.int32, device=dev),
                    cu_q=torch.tensor([0, T], dtype=torch.int32, device=dev), max_q=T, max_seq_len=T,
                    logits_idx=pos)
    return m.forward(tokens, meta, cache).float()


@pytest.mark.gpu
def test_lm_forward_matches_fused_kernels_and_merged_lora():
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel
    from axropus_deploy_b200.policy.local_model import LoRA, LocalReasoningModel, lm_forward

    m = LlamaModel(get_config("tiny128"), "cuda", seed=3, init_std=0.05)
    dev = torch.device("cuda", 0)
    toks = torch.arange(7, 7 + 200, dtype=torch.int32, device=dev) * 37 % m.cfg.vocab
    fused = _fused_logits(m, toks)
    ref = lm_forward(m, toks.long())
    assert float((fused - ref).norm() / ref.norm()) < 2e-2

    lora = LoRA(m, r=8)
    with torch.no_grad():
        for p in lora.B.values():
            p.normal_(0, 0.02)
    adapted = lm_forward(m, toks.long(), lora)
    assert float((adapted - ref).norm() / ref.norm()) > 2e-2
    lora.merge()  # the fused kernels now serve the adapted model
    fused2 = _fused_logits(m, toks)
    assert float((fused2 - adapted).norm() / adapted.norm()) < 2e-2
    lora.unmerge()

    lm = LocalReasoningModel(m, lora=lora, max_prompt_tokens=64)
    d = lm.decide(np.linspace(0, 1, 72, dtype=np.float32))
    assert not d.validate()
