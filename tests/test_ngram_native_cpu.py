"""Native incremental n-gram index (csrc/native/ngram.cpp) against the stateless scan of
:class:`NgramDrafter.propose`: random sequences with repeats, every n range, skip and
window, fed one step at a time as a decode would."""
from types import SimpleNamespace

import numpy as np
import pytest

from axropus_deploy_b200.engine.spec import NgramDrafter


@pytest.mark.parametrize("max_n,min_n,window,skip", [(3, 1, 4096, 0), (3, 1, 4096, 1), (6, 4, 4096, 0),
                                                     (3, 1, 37, 0), (2, 2, 64, 2)])
def test_index_matches_scan(max_n, min_n, window, skip):
    rng = np.random.default_rng(max_n * 100 + window + skip)
    for trial in range(6):
        vocab = int(rng.choice([3, 8, 50]))
        prompt = rng.integers(0, vocab, int(rng.integers(1, 300))).tolist()
        r = SimpleNamespace(req_id=f"r{trial}", prompt=prompt, output=[int(rng.integers(0, vocab))])
        d = NgramDrafter(max_n, min_n, window, skip)
        for _ in range(40):
            k = int(rng.integers(1, 9))
            assert d.propose_req(r, k) == d.propose(r.prompt + r.output, k)
            # accept a few tokens, sometimes the proposal itself (as verification would)
            step = d.propose(r.prompt + r.output, k)[: int(rng.integers(0, k + 1))] + [int(rng.integers(0, vocab))]
            r.output += step
        d.forget(r.req_id)
        assert r.req_id not in d._tables


def test_long_prompt_indexes_only_the_window():
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, 20, 20000).tolist()
    r = SimpleNamespace(req_id="long", prompt=prompt, output=[3])
    d = NgramDrafter(3, 1, 512)
    assert d.propose_req(r, 5) == d.propose(prompt + [3], 5)
    assert len(d._tables["long"][0]) <= 512 + 3 + 1
    r.output += [4, 5, 6]
    assert d.propose_req(r, 5) == d.propose(r.prompt + r.output, 5)
    # a shorter sequence under the same id (a reused id) rebuilds the index
    r2 = SimpleNamespace(req_id="long", prompt=prompt[:100], output=[1])
    assert d.propose_req(r2, 4) == d.propose(r2.prompt + r2.output, 4)
