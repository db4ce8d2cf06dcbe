"""The headline bench's request stream: every rank draws the same global wave and keeps its
routed share; cold prefills stay balanced over waves; replaying the choice state repeats the
mix (CPU, no GPU)."""
import hashlib
import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


def _owner(world):
    return lambda toks: int(hashlib.blake2b(str(toks[:8]).encode(), digest_size=4).hexdigest(), 16) % world


@pytest.mark.parametrize("world", [1, 2, 8])
def test_waves_partition_and_balance(world):
    args = bench.parse_args(["--prefix-len", "16", "--suffix-len", "4", "--batch", "32"])
    wls = [bench.Workload(args, 1000, r, world, _owner(world)) for r in range(world)]
    cold_total = [0] * world
    for _ in range(6):
        shares = [wl.wave(args.batch) for wl in wls]
        assert all(len(s) == args.batch for s in shares)
        allp = [tuple(p) for s in shares for p in s]
        assert len(set(allp)) == len(allp) == world * args.batch  # a partition of the global wave
        known = {tuple(p) for p in wls[0].prefixes}
        for r, s in enumerate(shares):
            cold_total[r] += sum(tuple(p[:16]) not in known for p in s)
    assert max(cold_total) - min(cold_total) <= 1
    # 10 % of 6 waves x world x 32 requests are cold, spread over the GPUs
    assert sum(cold_total) == pytest.approx(0.1 * 6 * world * 32, abs=1)
    assert all(wl.cold_carry == wls[0].cold_carry for wl in wls)


def test_choice_state_replays_the_mix():
    args = bench.parse_args(["--prefix-len", "16", "--suffix-len", "4"])
    wl = bench.Workload(args, 1000, 0, 1)
    known = {tuple(p) for p in wl.prefixes}
    st = wl.choice_state()
    a = wl.wave(32)
    wl.set_choice_state(st)
    b = wl.wave(32)
    # the same pooled prefixes at the same positions; fresh prefixes and suffixes get new tokens
    kind = lambda w: [tuple(p[:16]) if tuple(p[:16]) in known else "fresh" for p in w]  # noqa: E731
    assert kind(a) == kind(b) and "fresh" in kind(a)
    assert [p[16:] for p in a] != [p[16:] for p in b]
