"""Owner-affinity routing of a data-parallel wave (parallel/dp_router.py)."""
import random

from axropus_deploy_b200.parallel.dp_router import route_wave, routing_stats


def test_balanced_and_owner_first():
    rnd = random.Random(0)
    world, per = 8, 32
    owners = [min(7, int(rnd.paretovariate(1.1))) % world for _ in range(world * per)]  # skewed owners
    cold = [i % 10 == 0 for i in range(world * per)]
    a = route_wave(owners, cold, world, per)
    assert all(a.count(r) == per for r in range(world))  # weak scaling: equal work
    n_cold = [sum(1 for i in range(len(a)) if cold[i] and a[i] == r) for r in range(world)]
    assert max(n_cold) - min(n_cold) <= 1  # cold prefills spread evenly
    st = routing_stats(owners, cold, a)
    # every owner keeps as many of its own pooled requests as its capacity allows
    for r in range(world):
        own = [i for i in range(len(a)) if not cold[i] and owners[i] == r]
        kept = sum(1 for i in own if a[i] == r)
        assert kept == len(own) or sum(1 for x in a if x == r) == per
    assert 0 < st["miss_share"] < 1
    assert a == route_wave(owners, cold, world, per)  # deterministic: every rank computes the same


def test_single_gpu_and_capacity_check():
    assert route_wave([3, 1, 2], [False, True, False], 1, 3) == [0, 0, 0]
    try:
        route_wave([0] * 10, [False] * 10, 2, 4)
    except ValueError:
        pass
    else:
        raise AssertionError("capacity below the wave size must be refused")


def test_cold_remainders_balanced_over_waves():
    """Waves whose cold requests do not divide evenly: with the carried counts, no GPU
    collects every remainder, the cumulative cold prefills stay within one of each other."""
    import random

    rng = random.Random(3)
    world, per = 4, 8
    carry = [0] * world
    for _ in range(25):
        n_cold = rng.choice([2, 3, 5])
        cold = [True] * n_cold + [False] * (world * per - n_cold)
        owners = [rng.randrange(world) for _ in cold]
        a = route_wave(owners, cold, world, per, carry)
        assert all(sum(1 for r in a if r == q) <= per for q in range(world))
        assert max(carry) - min(carry) <= 1
