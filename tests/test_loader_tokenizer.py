"""Real-model serving pieces on CPU: Hugging Face checkpoints (models/loader.py) against
the transformers implementation of the same weights, and the tokenizer.json BPE
(models/tokenizer.py) against the tokenizers library on tokenizers trained here."""
import json
import os
import random

import pytest
import torch

from axropus_deploy_b200.models.loader import load_pretrained, read_config, save_pretrained
from axropus_deploy_b200.models.tokenizer import Tokenizer


def _hf_llama(tmp_path):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.LlamaConfig(vocab_size=1000, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=2048,
                                   rope_theta=500000.0, rms_norm_eps=1e-5, tie_word_embeddings=False,
                                   rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                                 "high_freq_factor": 4.0, "original_max_position_embeddings": 256})
    torch.manual_seed(0)
    m = transformers.LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    d = str(tmp_path / "hf")
    m.save_pretrained(d, safe_serialization=True)
    return m, d


def test_checkpoint_matches_transformers_forward(tmp_path):
    from axropus_deploy_b200.models.llama import AttnMeta
    from axropus_deploy_b200.ops.kvcache import KVCache

    hf, d = _hf_llama(tmp_path)
    mc, _ = read_config(d)
    assert (mc.num_layers, mc.hidden, mc.num_kv_heads, mc.head_dim) == (2, 512, 2, 128)
    ours = load_pretrained(d, "cpu")
    T = 40
    toks = torch.randint(0, 1000, (T,))
    with torch.no_grad():
        ref = hf(toks[None]).logits[0].float()
    cache = KVCache(2, 8, 2, 128, "bf16", "cpu")
    pos = torch.arange(T, dtype=torch.int32)
    meta = AttnMeta(mode="prefill", positions=pos, slots=pos.clone(), block_table=torch.arange(8, dtype=torch.int32)[None],
                    seq_lens=torch.tensor([T], dtype=torch.int32), cu_q=torch.tensor([0, T], dtype=torch.int32),
                    max_q=T, max_seq_len=T, logits_idx=torch.arange(T, dtype=torch.int32))
    got = ours.forward(toks.to(torch.int32), meta, cache).float()
    # bf16 weights and activations on both sides: compare the distributions and the argmax
    cos = torch.nn.functional.cosine_similarity(got, ref, dim=-1)
    assert cos.min().item() > 0.99, cos
    assert (got.argmax(-1) == ref.argmax(-1)).float().mean().item() >= 0.9


def test_save_load_round_trip_dense_and_moe(tmp_path):
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    for name in ("tiny128", "tiny-moe"):
        m = LlamaModel(get_config(name), "cpu", seed=5)
        d = str(tmp_path / name)
        save_pretrained(m, d)
        m2 = load_pretrained(d, "cpu")
        for a, b in zip(m.layers, m2.layers):
            for f in ("wqkv", "wo", "w_gate_up", "w_down", "w_router", "w13", "w2", "attn_norm", "mlp_norm"):
                x, y = getattr(a, f), getattr(b, f)
                assert (x is None) == (y is None) and (x is None or torch.equal(x, y)), f
        assert torch.equal(m.lm_head, m2.lm_head) and torch.equal(m.embed, m2.embed)


# ----------------------------------------------------------------------------- tokenizer
def _corpus(n=3000, seed=0):
    rnd = random.Random(seed)
    words = ["the", "cache", "prefix", "restore", "token", "GPU", "Blackwell", "naïve", "déjà", "vu", "東京", "🙂",
             "42", "1234567", "don't", "we'll", "x=y+1;", "\n", "  ", "\t"]
    return [" ".join(rnd.choice(words) for _ in range(rnd.randint(3, 12))) for _ in range(n)]


def _samples(seed=1):
    rnd = random.Random(seed)
    alphabet = "abcdefg ,.!?'0123456789\n\té東京🙂<>|_-"
    out = ["", " ", "hello world", "don't stop", "  leading spaces", "tabs\tand\nnewlines\n\n", "東京🙂 naïve",
           "<|begin_of_text|>hi<|eot_id|>", "12345678901", "x=y+1; z=\"q\""]
    out += ["".join(rnd.choice(alphabet) for _ in range(rnd.randint(1, 40))) for _ in range(200)]
    return out


def test_byte_level_bpe_matches_tokenizers_library(tmp_path):
    tk = pytest.importorskip("tokenizers")
    from tokenizers import Regex, decoders, models, pre_tokenizers, trainers

    split = r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"
    t = tk.Tokenizer(models.BPE(ignore_merges=True))
    t.pre_tokenizer = pre_tokenizers.Sequence([pre_tokenizers.Split(Regex(split), "isolated"),
                                               pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    t.decoder = decoders.ByteLevel()
    t.train_from_iterator(_corpus(), trainers.BpeTrainer(vocab_size=600, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                                         special_tokens=["<|begin_of_text|>", "<|eot_id|>"]))
    path = str(tmp_path / "tokenizer.json")
    t.save(path)
    ours = Tokenizer.from_file(path)
    for s in _samples():
        want = t.encode(s, add_special_tokens=False).ids
        assert ours.encode(s) == want, s
        assert ours.decode(want, skip_special_tokens=False) == t.decode(want, skip_special_tokens=False), s


def test_metaspace_byte_fallback_bpe_matches_tokenizers_library(tmp_path):
    tk = pytest.importorskip("tokenizers")
    from tokenizers import decoders, models, pre_tokenizers, trainers

    t = tk.Tokenizer(models.BPE(byte_fallback=True, unk_token="<unk>", fuse_unk=True))
    t.pre_tokenizer = pre_tokenizers.Metaspace(replacement="▁", prepend_scheme="first")
    t.decoder = decoders.Sequence([decoders.Replace("▁", " "), decoders.ByteFallback(), decoders.Fuse(),
                                   decoders.Strip(" ", 1, 0)])
    specials = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    t.train_from_iterator(_corpus(seed=3), trainers.BpeTrainer(vocab_size=700, special_tokens=specials,
                                                               limit_alphabet=60))
    path = str(tmp_path / "tokenizer.json")
    t.save(path)
    ours = Tokenizer.from_file(path)
    for s in _samples(seed=2):
        if "<" in s:  # the byte tokens are added tokens of this test tokenizer: keep them out of the text
            continue
        want = t.encode(s, add_special_tokens=False).ids
        assert ours.encode(s) == want, s
        assert ours.decode(want) == t.decode(want), s


def test_server_serves_checkpoint_with_its_tokenizer(tmp_path):
    tk = pytest.importorskip("tokenizers")
    from fastapi.testclient import TestClient
    from tokenizers import decoders, models, pre_tokenizers, trainers

    from axropus_deploy_b200.config import AxropusConfig, KorithConfig
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel
    from axropus_deploy_b200.server.app import build_engine, create_app

    d = str(tmp_path / "model")
    save_pretrained(LlamaModel(get_config("tiny128"), "cpu", seed=7), d)
    t = tk.Tokenizer(models.BPE())
    t.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    t.decoder = decoders.ByteLevel()
    t.train_from_iterator(_corpus(), trainers.BpeTrainer(vocab_size=500, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                                         special_tokens=["<|begin_of_text|>", "<|start_header_id|>",
                                                                         "<|end_header_id|>", "<|eot_id|>"]))
    t.save(os.path.join(d, "tokenizer.json"))
    cfg = AxropusConfig(model=d, device="cpu")
    k = KorithConfig()
    k.enable_amf = False
    k.vram_cache_gb = 0.05
    k.n_ctx = 2048
    eng = build_engine(cfg, k, num_blocks=128)
    with TestClient(create_app(cfg, eng)) as c:
        assert c.get("/healthz").json()["tokenizer"] == "tokenizer.json"
        r = c.post("/v1/completions", json={"prompt": "the cache prefix restore token", "max_tokens": 3}).json()
        assert r["usage"]["prompt_tokens"] == len(t.encode("the cache prefix restore token").ids)
        assert r["choices"][0]["text"] == t.decode(r["token_ids"])
        r2 = c.post("/v1/chat/completions", json={"messages": [{"role": "user", "content": "hi"}],
                                                  "max_tokens": 2}).json()
        assert r2["usage"]["completion_tokens"] == 2 and r2["usage"]["prompt_tokens"] > 5
