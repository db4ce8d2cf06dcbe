"""Mixed steps on the GPU: one forward over new prompts' tokens and one decode token per
running sequence gives the logits of a separate prefill forward and a separate decode
forward (fp32 comparison of bf16 logits), through the tcgen05 projections, the prefill
attention kernel and the split-KV decode kernel; and the engine takes the mixed path when
prompts are admitted while others decode."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _meta_prefill(prompts, starts, blocks, dev):
    from axropus_deploy_b200.models.llama import AttnMeta

    toks, pos, slots, cu, lens = [], [], [], [0], []
    for p, s0, b in zip(prompts, starts, blocks):
        for i in range(s0, len(p)):
            toks.append(p[i])
            pos.append(i)
            slots.append(b[i // 16] * 16 + i % 16)
        cu.append(cu[-1] + len(p) - s0)
        lens.append(len(p))
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    width = max(len(b) for b in blocks)
    bt = i32([b + [0] * (width - len(b)) for b in blocks])
    meta = AttnMeta(mode="prefill", positions=i32(pos), slots=i32(slots), block_table=bt, seq_lens=i32(lens),
                    cu_q=i32(cu), max_q=max(cu[i + 1] - cu[i] for i in range(len(prompts))), max_seq_len=max(lens),
                    logits_idx=i32([c - 1 for c in cu[1:]]))
    return toks, meta


def test_mixed_forward_matches_separate_forwards():
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import AttnMeta, LlamaModel
    from axropus_deploy_b200.ops.kvcache import KVCache

    dev = torch.device("cuda", 0)
    cfg = get_config("tiny128")
    model = LlamaModel(cfg, dev, seed=0)
    cache = KVCache(cfg.num_layers, 256, cfg.num_kv_heads, cfg.head_dim, "bf16", dev)
    g = torch.Generator().manual_seed(11)
    rnd = lambda n: torch.randint(0, cfg.vocab, (n,), generator=g).tolist()  # noqa: E731
    # three sequences already prefilled (they decode), two new prompts (one over a cached prefix)
    old = [rnd(n) for n in (300, 517, 64)]
    new = [rnd(n) for n in (200, 400)]
    nb = 0
    blocks = []
    for p in old + new:
        k = (len(p) + 1 + 15) // 16
        blocks.append(list(range(nb, nb + k)))
        nb += k
    i32 = lambda x: torch.tensor(x, dtype=torch.int32, device=dev)  # noqa: E731
    toks, meta = _meta_prefill(old, [0, 0, 0], blocks[:3], dev)
    model.forward(i32(toks), meta, cache)
    # new prompt 1 reuses a cached prefix of 128 tokens: prefill its first 128 first
    toks, meta = _meta_prefill([new[1][:128]], [0], [blocks[4]], dev)
    model.forward(i32(toks), meta, cache)
    starts = [0, 128]
    # decode inputs: one token per old sequence at position len(p)
    dtok = rnd(3)
    dpos = [len(p) for p in old]
    dslots = [blocks[i][dpos[i] // 16] * 16 + dpos[i] % 16 for i in range(3)]
    dlens = [p_ + 1 for p_ in dpos]
    width = max(len(b) for b in blocks)
    dbt = i32([b + [0] * (width - len(b)) for b in blocks[:3]])
    dmeta = AttnMeta(mode="decode", positions=i32(dpos), slots=i32(dslots), block_table=dbt, seq_lens=i32(dlens),
                     max_seq_len=max(dlens))
    # separate forwards
    ptoks, pmeta = _meta_prefill(new, starts, blocks[3:], dev)
    ref_p = model.forward(i32(ptoks), pmeta, cache).float()
    ref_d = model.forward(i32(dtok), dmeta, cache).float()
    # one mixed forward over the same rows (it rewrites the same KV slots)
    tp = len(ptoks)
    mmeta = AttnMeta(mode="mixed", positions=torch.cat([pmeta.positions, dmeta.positions]),
                     slots=torch.cat([pmeta.slots, dmeta.slots]), block_table=pmeta.block_table,
                     seq_lens=pmeta.seq_lens, cu_q=pmeta.cu_q, max_q=pmeta.max_q, max_seq_len=pmeta.max_seq_len,
                     logits_idx=torch.cat([pmeta.logits_idx, i32(list(range(tp, tp + 3)))]), decode=dmeta)
    out = model.forward(i32(ptoks + dtok), mmeta, cache).float()
    torch.cuda.synchronize()
    for got, want in ((out[:2], ref_p), (out[2:], ref_d)):
        err = (got - want).abs().max().item() / (want.abs().max().item() + 1e-6)
        assert err < 2e-2, err


def test_engine_takes_mixed_steps():
    from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    dev = torch.device("cuda", 0)
    cfg = get_config("tiny128")
    model = LlamaModel(cfg, dev, seed=0)
    eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024, max_batch=8, max_prefill_tokens=300,
                                        cuda_graphs=True))
    g = torch.Generator().manual_seed(3)
    reqs = [eng.add_request(torch.randint(0, cfg.vocab, (n,), generator=g).tolist(), SamplingParams(max_tokens=8))
            for n in (250, 260, 270, 280)]
    while eng.has_unfinished():
        eng.step()
    eng.close()
    assert eng.stat["mixed_steps"] > 0
    assert all(len(r.output) == 8 for r in reqs)
