"""bench.py's config-4 leg: the 8 seeded uneven shards (10-20% of 229,376 positions each, the draw of
tests/test_configs_gpu.py) and their grouping onto 1, 2, 4 and 8 ranks as contiguous position ranges."""
import numpy as np

import bench
from backburner_b200 import shard


def test_uneven_shares_match_the_config4_draw_and_group_onto_the_ranks():
    rng = np.random.default_rng(41)
    w = rng.uniform(0.10, 0.20, 8)
    eight = np.floor(w / w.sum() * 229376).astype(int)
    eight[-1] += 229376 - eight.sum()
    assert bench.uneven_shares(8) == [int(x) for x in eight]
    for world in (1, 2, 4, 8):
        shares = bench.uneven_shares(world)
        assert len(shares) == world and sum(shares) == bench.U_KEYS
        per = 8 // world
        assert shares == [int(eight[r * per:(r + 1) * per].sum()) for r in range(world)]
        # the ranks' position ranges are contiguous, in rank order
        starts = [shard.shard_range(bench.U_KEYS, world, r, shares)[0] for r in range(world)]
        assert starts == [sum(shares[:r]) for r in range(world)]
    # weights drawn from [0.10, 0.20): the smallest shard is at least about half the largest
    assert min(eight) > 0.5 * max(eight) * 0.99
