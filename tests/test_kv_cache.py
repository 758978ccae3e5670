"""The sharded KV cache's host logic on CPU: which rank stores which appended
tokens (scope_b200.kv_cache.local_slice / shard_capacity), checked against a
plain per-position assignment for prefill chunks and single-token steps."""
import pytest

from scope_b200.kv_cache import local_slice, shard_capacity


@pytest.mark.parametrize("max_seq,world", [(10, 1), (10, 3), (16, 4), (7, 8), (131072, 8)])
def test_appends_land_on_the_owning_rank(max_seq, world):
    cap = shard_capacity(max_seq, world)
    assert cap * world >= max_seq and cap * (world - 1) < max_seq or world == 1 or max_seq < world
    owner = {}
    t = 0
    steps = [min(5, max_seq)] + [1] * (min(max_seq, 40) - min(5, max_seq))
    for n in steps:
        seen = 0
        for r in range(world):
            first, cnt, t0 = local_slice(t, n, cap, r)
            for i in range(cnt):
                pos = t + first + i
                assert pos not in owner
                owner[pos] = (r, t0 + i)
                assert r * cap + t0 + i == pos and 0 <= t0 + i < cap
            seen += cnt
        assert seen == n
        t += n
    assert sorted(owner) == list(range(t))


def test_local_slice_edges():
    assert local_slice(0, 0, 4, 0) == (0, 0, 0)
    assert local_slice(3, 3, 4, 0) == (0, 1, 3)    # positions 3 | 4, 5
    assert local_slice(3, 3, 4, 1) == (1, 2, 0)
    assert local_slice(3, 3, 4, 2) == (0, 0, 0)
