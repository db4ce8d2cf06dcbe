"""Shared-prefix (cascade) decode attention: grouped sequences attend to their shared
pages in one tcgen05 pass and to their own pages in the split-KV decode kernel; the
merged result must equal plain decode attention and the fp32 CPU oracle. Also the
padded form the decode CUDA graphs replay (empty groups, padded rows)."""
import pytest
import torch

from axropus_deploy_b200.ops import KVCache, decode_attention
from axropus_deploy_b200.ops.attention import CascadeMeta, cascade_groups

pytestmark = pytest.mark.gpu


def _setup(seed=0):
    g = torch.Generator().manual_seed(seed)
    Hkv, G, D, NB = 2, 4, 128, 400
    cache = KVCache(1, NB, Hkv, D, "bf16", "cuda")
    cache.data.copy_(torch.randn(cache.data.shape, generator=g).to(torch.bfloat16))
    perm = torch.randperm(NB, generator=g).tolist()
    shared_a, shared_b = perm[:40], perm[40:75]
    free = perm[75:]
    lists, lens = [], []
    for i, (pref, own_tokens) in enumerate([(shared_a, 200), (shared_a, 37), (shared_a, 5), (shared_b, 99),
                                             (shared_b, 16), (None, 700)]):
        n_own = (own_tokens + 15) // 16
        own = [free.pop() for _ in range(n_own)]
        lists.append((pref or []) + own)
        lens.append((len(pref) * 16 if pref else 0) + own_tokens)
    B = len(lists)
    width = max(len(x) for x in lists) + 3
    bt = torch.zeros(B, width, dtype=torch.int32)
    for i, x in enumerate(lists):
        bt[i, :len(x)] = torch.tensor(x, dtype=torch.int32)
    q = torch.randn(B, Hkv * G, D, generator=g).to(torch.bfloat16)
    return cache, lists, bt.cuda(), torch.tensor(lens, dtype=torch.int32).cuda(), q.cuda()


def _meta(lists, bt, groups, B, pad_groups=0, max_q=None, splits=3):
    q_index, cu, slen, first = [], [0], [], []
    row_of, ps = [-1] * B, [0] * B
    for rows, shared in groups:
        for i in rows:
            row_of[i] = len(q_index)
            ps[i] = shared
            q_index.append(i)
        cu.append(len(q_index))
        slen.append(shared * 16)
        first.append(rows[0])
    cu += [cu[-1]] * pad_groups
    slen += [0] * pad_groups
    first += [0] * pad_groups
    dev = bt.device
    qi = torch.tensor(q_index + [0] * (B - len(q_index)), dtype=torch.int32, device=dev)
    return CascadeMeta(q_index=qi, cu_q=torch.tensor(cu, dtype=torch.int32, device=dev),
                       seq_lens=torch.tensor(slen, dtype=torch.int32, device=dev),
                       block_table=bt.index_select(0, torch.tensor(first, device=dev)),
                       row_of=torch.tensor(row_of, dtype=torch.int32, device=dev),
                       page_start=torch.tensor(ps, dtype=torch.int32, device=dev),
                       max_q=max_q or max(len(r) for r, _ in groups), num_splits=splits)


def _oracle(cache, bt, sl, q):
    c = KVCache(1, cache.num_blocks, cache.num_kv_heads, 128, "bf16", "cpu")
    c.data.copy_(cache.data.cpu())
    return decode_attention(q.cpu(), c, 0, bt.cpu(), sl.cpu())


@pytest.mark.parametrize("splits", [1, 3, 8])
def test_cascade_matches_plain_decode(splits):
    cache, lists, bt, sl, q = _setup()
    groups = cascade_groups(lists, min_pages=32, max_pages=[int(x) // 16 for x in sl.tolist()])
    assert sorted((tuple(r), s) for r, s in groups) == [((0, 1, 2), 40), ((3, 4), 35)]
    max_seq = int(sl.max())
    plain = decode_attention(q, cache, 0, bt, sl, max_seq_len=max_seq)
    casc = decode_attention(q, cache, 0, bt, sl, max_seq_len=max_seq, cascade=_meta(lists, bt, groups, q.shape[0],
                                                                                     splits=splits))
    torch.cuda.synchronize()
    torch.testing.assert_close(casc.float(), plain.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(casc.float().cpu(), _oracle(cache, bt, sl, q).float(), atol=2e-2, rtol=2e-2)


def test_cascade_padded_graph_form():
    """As the decode graphs replay it: max_q = batch, group slots beyond the real groups
    empty, a padded batch row with length 0."""
    cache, lists, bt, sl, q = _setup(1)
    groups = cascade_groups(lists, min_pages=32)
    B = q.shape[0]
    qp = torch.cat([q, torch.zeros_like(q[:1])])
    btp = torch.cat([bt, torch.zeros_like(bt[:1])])
    slp = torch.cat([sl, torch.zeros_like(sl[:1])])
    m = _meta(lists, btp, groups, B + 1, pad_groups=(B + 1) // 2 - len(groups), max_q=B + 1, splits=4)
    casc = decode_attention(qp, cache, 0, btp, slp, max_seq_len=int(sl.max()) + 64, num_splits=5, cascade=m)
    plain = decode_attention(q, cache, 0, bt, sl, max_seq_len=int(sl.max()))
    torch.cuda.synchronize()
    torch.testing.assert_close(casc[:B].float(), plain.float(), atol=2e-2, rtol=2e-2)
    assert casc[B].abs().max().item() == 0.0


def test_cascade_no_groups_is_plain():
    cache, lists, bt, sl, q = _setup(2)
    B = q.shape[0]
    dev = bt.device
    empty = CascadeMeta(q_index=torch.zeros(B, dtype=torch.int32, device=dev),
                        cu_q=torch.zeros(4, dtype=torch.int32, device=dev),
                        seq_lens=torch.zeros(3, dtype=torch.int32, device=dev), block_table=bt[:3],
                        row_of=torch.full((B,), -1, dtype=torch.int32, device=dev),
                        page_start=torch.zeros(B, dtype=torch.int32, device=dev), max_q=B, num_splits=2)
    casc = decode_attention(q, cache, 0, bt, sl, max_seq_len=int(sl.max()), cascade=empty)
    plain = decode_attention(q, cache, 0, bt, sl, max_seq_len=int(sl.max()))
    torch.cuda.synchronize()
    torch.testing.assert_close(casc.float(), plain.float(), atol=1e-2, rtol=1e-2)
