"""vLLM v1 KV connector over the AMF prefix keys (axropus_deploy_b200.amf.vllm_connector),
driven on CPU with stand-ins for vLLM's config, requests and scheduler output: a cold
request's block-aligned prefix is saved layer by layer, a later request with the same prefix
is told the prefix is loadable, and the load writes those pages into its own blocks."""
from types import SimpleNamespace

import pytest
import torch

vllm_base = pytest.importorskip("vllm.distributed.kv_transfer.kv_connector.v1.base")


def _cfg(eid):
    return SimpleNamespace(kv_transfer_config=SimpleNamespace(kv_connector_extra_config={"pool_gb": 0.01,
                                                                                         "min_prefix_tokens": 16},
                                                              engine_id=eid),
                           cache_config=SimpleNamespace(block_size=16))


class _Blocks:
    def __init__(self, ids):
        self.ids = ids

    def get_block_ids(self):
        return (self.ids,)


@pytest.mark.parametrize("layout", ["flash", "blocks_first"])
def test_connector_save_then_load(layout):
    from axropus_deploy_b200.amf.vllm_connector import AMFKVConnector, AmfB200Connector

    assert AMFKVConnector is AmfB200Connector
    role = vllm_base.KVConnectorRole
    sched = AmfB200Connector(_cfg("t-" + layout), role.SCHEDULER)
    work = AmfB200Connector(_cfg("t-" + layout), role.WORKER)
    g = torch.Generator().manual_seed(0)
    shape = (2, 64, 16, 2, 8) if layout == "flash" else (64, 2, 16, 2, 8)
    caches = {f"model.layers.{i}.attn": torch.randn(*shape, generator=g) for i in range(3)}
    work.register_kv_caches(caches)
    prefix = torch.randint(0, 1000, (64,), generator=g).tolist()
    a_toks = prefix + [1, 2, 3, 4, 5, 6]
    # step 1: request A prefills cold; its 64-token prefix (blocks 5, 9, 2, 7) is saved
    req_a = SimpleNamespace(request_id="A", prompt_token_ids=a_toks)
    assert sched.get_num_new_matched_tokens(req_a, 0) == (0, False)
    out1 = SimpleNamespace(scheduled_new_reqs=[SimpleNamespace(req_id="A", prompt_token_ids=a_toks,
                                                               block_ids=([5, 9, 2, 7, 11],), num_computed_tokens=0)],
                           num_scheduled_tokens={"A": len(a_toks)})
    meta = sched.build_connector_meta(out1)
    assert len(meta.saves) == 1 and meta.saves[0].block_ids == [5, 9, 2, 7] and not meta.loads
    work.bind_connector_metadata(meta)
    work.start_load_kv(None)
    for name, kv in caches.items():
        work.save_kv_layer(name, kv, None)
    work.wait_for_save()
    work.clear_connector_metadata()
    assert sched.store.stat["saves"] == 1
    # step 2: request B shares the prefix; 64 tokens are loadable into its blocks 20..23
    b_toks = prefix + list(range(900, 916))
    req_b = SimpleNamespace(request_id="B", prompt_token_ids=b_toks)
    assert sched.get_num_new_matched_tokens(req_b, 0) == (64, False)
    sched.update_state_after_alloc(req_b, _Blocks([20, 21, 22, 23, 24]), 64)
    out2 = SimpleNamespace(scheduled_new_reqs=[SimpleNamespace(req_id="B", prompt_token_ids=b_toks,
                                                               block_ids=([20, 21, 22, 23, 24],), num_computed_tokens=64)],
                           num_scheduled_tokens={"B": 16})
    meta2 = sched.build_connector_meta(out2)
    assert len(meta2.loads) == 1 and not meta2.saves  # the prefix is already held
    before = {n: kv.clone() for n, kv in caches.items()}
    work.bind_connector_metadata(meta2)
    work.start_load_kv(None)
    work.clear_connector_metadata()
    d = 1 if layout == "flash" else 0
    for n, kv in caches.items():
        got = kv.index_select(d, torch.tensor([20, 21, 22, 23]))
        want = before[n].index_select(d, torch.tensor([5, 9, 2, 7]))
        assert torch.equal(got, want)
    # a prompt sharing only the first 32 tokens loads those two blocks
    part = prefix[:32] + list(range(500, 560))
    req_p = SimpleNamespace(request_id="P", prompt_token_ids=part)
    assert sched.get_num_new_matched_tokens(req_p, 0) == (32, False)
    # a prompt whose first 16 tokens differ matches nothing
    other = SimpleNamespace(request_id="C", prompt_token_ids=[7] * 80)
    assert sched.get_num_new_matched_tokens(other, 0) == (0, False)
