"""The N>1 host path on CPU: world-size-2 gloo ranks each compute the oracle's partial over their position shard, pack
it as pa_cuda_merge_gathered expects, exchange with one all-gather, and fold; the result equals the partial over all
positions. Equal and uneven (config 4 style) shares, and a rank with no positions."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from backburner_b200 import shard


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, n_keys, shares, q):
    import torch
    import torch.distributed as dist
    from oracle import oracle as orc
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        c = orc.gen_case(7, 128, 4, 5, n_keys, orc.Q8_0)          # same seeded case on every rank
        start, count = shard.shard_range(n_keys, world, rank, shares)
        O, m, l = orc.partial_f32(c["shape"], c["Qs"], c["K"][start:start + count], c["V"][start:start + count], count)
        rows = 4 * 5
        if count == 0:
            m[:] = -np.inf
        buf = torch.from_numpy(shard.pack(O.reshape(rows, 128), m.reshape(rows), l.reshape(rows)))
        gathered = torch.empty((world * buf.numel(),), dtype=buf.dtype)
        dist.all_gather_into_tensor(gathered, buf)
        gathered = gathered.view(world, -1)
        parts = [shard.unpack(gathered[r].numpy(), rows, 128) for r in range(world)]
        Om, mm, lm = orc.merge_slots(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]),
                                     np.stack([p[2] for p in parts]))
        Ow, mw, lw = orc.partial_f32(c["shape"], c["Qs"], c["K"], c["V"], n_keys)
        e = orc.rel_err(Om, mm, lm, Ow.reshape(rows, 128).astype(np.float64), mw.reshape(rows).astype(np.float64),
                        lw.reshape(rows).astype(np.float64))
        q.put((rank, e))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_keys,shares", [(3000, None), (3001, None), (3000, [400, 2600]), (1000, [0, 1000])])
def test_two_rank_shards_fold_to_the_whole(n_keys, shares):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, n_keys, shares, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict(q.get(timeout=5) for _ in range(2))
    for r in range(2):
        eo, el = res[r]
        assert eo < 5e-4 and el < 1e-5, (r, eo, el)


def test_shard_ranges():
    assert shard.shard_range(131072, 8, 0) == (0, 16384)
    assert shard.shard_range(131073, 8, 7) == (7 * 16384, 16385)
    assert sum(shard.shard_range(229376, 8, r, [30000] * 7 + [19376])[1] for r in range(8)) == 229376
    with pytest.raises(ValueError):
        shard.shard_range(10, 2, 0, [3, 3])
