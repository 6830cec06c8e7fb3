"""pa_cuda_shard_attn_allgather_merge: position shards over NCCL in one call (one process per GPU; each rank's plan covers
its contiguous range of positions of every output set; the ranks' packed (O, m, l) are exchanged and folded on every
rank). Every exchange is covered: the all-gather followed by the fold, the max / sum all-reduces (with and without
output-set groups, a group's exchange overlapping the next group's kernels), and the peer stores over NVLink (each rank's
merged rows stored into every rank's receive buffer, the fold waiting on per-source counters).

A communicator of one rank must give what the plan alone gives; two ranks on two GPUs must agree with each other bit
for bit and with the oracle over all positions (2e-3, as the other parity tests). A rank that leaves between steps must
make the other rank's next bounded exchange fail (PA_CUDA_ETIMEOUT, or PA_CUDA_ENCCL when NCCL notices first) within
the bound, with its context still usable (NVLS off, plain peer transport, as the failure-detection tests on this pool
require). The multi-rank tests need two GPUs."""
import os
import time

import numpy as np
import pytest

import backburner_b200 as pa
from oracle import oracle as orc

from test_decode_gpu import TOL_REF

pytestmark = pytest.mark.gpu

HD, NKV, ROWS, NK, SETS = 128, 8, 5, 3000, 4
MODES = [(1, 1), (1, 3), (2, 1), (2, 3), (3, 1)]   # (exchange: 1 all-gather, 2 all-reduce, 3 peer stores; set groups)


def _cases():
    """One seeded case per output set (a layer each), the same on every rank."""
    return [orc.gen_case(62 + s, HD, NKV, ROWS, NK, orc.Q8_0) for s in range(SETS)]


def _inputs(torch, pa_mod, cases, dev, a, b):
    """Keys [a, b) of every set on `dev`, the stacked Q of all sets and the plan's segments."""
    K = [torch.from_numpy(np.ascontiguousarray(c["K"][a:b])).to(dev) for c in cases]
    V = [torch.from_numpy(np.ascontiguousarray(c["V"][a:b])).to(dev) for c in cases]
    Qs = torch.from_numpy(np.stack([c["Qs"] for c in cases]).view(np.int16)).to(dev).view(torch.float16)
    segs = [pa_mod.Seg(K[s].data_ptr(), V[s].data_ptr(), b - a, s) for s in range(SETS) if b > a]
    return K, V, Qs, segs


def test_one_rank_equals_the_plan(ctx):
    import torch
    cases = _cases()
    shape = pa.shape_for(HD, NKV, ROWS, pa.Q8_0)
    K, V, Qs, segs = _inputs(torch, pa, cases, torch.device("cuda", 0), 0, NK)
    plan = pa.Plan(ctx, shape, SETS, segs)
    O1 = torch.empty((SETS, NKV, ROWS, HD), device="cuda")
    m1 = torch.empty((SETS, NKV, ROWS), device="cuda")
    l1 = torch.empty_like(m1)
    plan.run(Qs, O1, m1, l1)
    comm = pa.NcclComm(ctx, pa.nccl_unique_id(), 0, 1)
    try:
        for mode, groups in MODES:
            ctx.set_shard_exchange(mode)
            ctx.set_shard_groups(groups)
            for _ in range(2):
                O2, m2, l2 = torch.full_like(O1, 7.0), torch.full_like(m1, 7.0), torch.full_like(l1, 7.0)
                pa.shard_attn_allgather_merge(plan, Qs, comm, O2, m2, l2)
                ctx.status()
                assert ctx.shard_last()[0] == mode, (mode, ctx.shard_last())
                # the same arithmetic up to the order of the fp32 sums (merges of different shapes)
                o1 = O1.cpu().numpy()
                np.testing.assert_allclose(O2.cpu().numpy(), o1, rtol=1e-5, atol=1e-6 * np.abs(o1).max())
                np.testing.assert_allclose(m2.cpu().numpy(), m1.cpu().numpy(), rtol=1e-6)
                np.testing.assert_allclose(l2.cpu().numpy(), l1.cpu().numpy(), rtol=1e-5)
    finally:
        ctx.set_shard_exchange(0)
        ctx.set_shard_groups(0)
        comm.close()
        plan.close()


def _rank(rank, world, uid, q):
    try:
        import torch
        import backburner_b200 as pa2
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        ctx = pa2.Context(rank)
        cases = _cases()
        a, b = rank * NK // world, (rank + 1) * NK // world
        shape = pa2.shape_for(HD, NKV, ROWS, pa2.Q8_0)
        K, V, Qs, segs = _inputs(torch, pa2, cases, dev, a, b)
        plan = pa2.Plan(ctx, shape, SETS, segs)
        comm = pa2.NcclComm(ctx, uid, rank, world)
        O = torch.empty((SETS, NKV, ROWS, HD), device=dev)
        m = torch.empty((SETS, NKV, ROWS), device=dev)
        l = torch.empty_like(m)
        out = {}
        ctx.set_shard_timeout_ms(60000)
        for mode, groups in MODES:
            ctx.set_shard_exchange(mode)
            ctx.set_shard_groups(groups)
            out[(mode, groups)] = []
            for _ in range(2):
                pa2.shard_attn_allgather_merge(plan, Qs, comm, O, m, l)
                ctx.status()
                assert ctx.shard_last()[0] == mode, (mode, ctx.shard_last())
                out[(mode, groups)].append((O.cpu().numpy(), m.cpu().numpy(), l.cpu().numpy()))
        comm.close()
        plan.close()
        ctx.close()
        q.put((rank, out, None))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def _spawn(target, world, *extra):
    import torch.multiprocessing as mp
    uid = pa.nccl_unique_id()
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    procs = [ctxm.Process(target=target, args=(r, world, uid, q, *extra)) for r in range(world)]
    for p in procs:
        p.start()
    return q, procs


def _join(procs):
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()


def test_two_ranks_on_two_gpus_match_the_oracle():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    q, procs = _spawn(_rank, 2)
    got = {}
    try:
        for _ in range(2):
            rank, out, err = q.get(timeout=300)
            assert err is None, (rank, err)
            got[rank] = out
    finally:
        _join(procs)
    refs = [orc.partial_f32(c["shape"], c["Qs"], c["K"], c["V"], NK) for c in _cases()]
    for key in got[0]:
        for rank in (0, 1):
            for O, m, l in got[rank][key]:
                for s, (Or, mr, lr) in enumerate(refs):
                    e = orc.rel_err(O[s], m[s], l[s], Or.astype(np.float64), mr.astype(np.float64),
                                    lr.astype(np.float64))
                    assert e[0] <= TOL_REF and e[1] <= TOL_REF, (key, rank, s, e)
                    assert np.abs(m[s] - mr).max() <= TOL_REF, (key, rank, s)
        # the fold is the same on every rank, bit for bit
        for i in range(2):
            for j in range(3):
                np.testing.assert_array_equal(got[0][key][i][j], got[1][key][i][j])


def _leaver(rank, world, uid, q, bound_ms):
    """Rank 1 takes one step and leaves (nothing of it in flight); rank 0's next step must fail within the bound."""
    try:
        import torch
        import backburner_b200 as pa2
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        ctx = pa2.Context(rank)
        cases = _cases()
        a, b = rank * NK // world, (rank + 1) * NK // world
        K, V, Qs, segs = _inputs(torch, pa2, cases, dev, a, b)
        plan = pa2.Plan(ctx, pa2.shape_for(HD, NKV, ROWS, pa2.Q8_0), SETS, segs)
        comm = pa2.NcclComm(ctx, uid, rank, world)
        O = torch.empty((SETS, NKV, ROWS, HD), device=dev)
        m = torch.empty((SETS, NKV, ROWS), device=dev)
        l = torch.empty_like(m)
        ctx.set_shard_timeout_ms(bound_ms)
        pa2.shard_attn_allgather_merge(plan, Qs, comm, O, m, l)   # step 1: both ranks, completed before returning
        ctx.status()
        if rank == 1:
            q.put((rank, "left", None))
            q.close()
            q.join_thread()                                       # the message is out before the process goes
            os._exit(0)                                           # between steps: nothing of this rank in flight
        time.sleep(1.0)                                           # the peer is gone before the next step
        t0 = time.time()
        try:
            pa2.shard_attn_allgather_merge(plan, Qs, comm, O, m, l)
            res = ("no error", time.time() - t0)
        except pa2.PaCudaError as e:
            res = (e.code, time.time() - t0)
        # the context stays usable: a plain plan run after the aborted exchange, checked against the oracle
        plan.run(Qs, O, m, l)
        ctx.status()
        Or, mr, lr = orc.partial_f32(cases[0]["shape"], cases[0]["Qs"], cases[0]["K"][a:b], cases[0]["V"][a:b], b - a)
        e = orc.rel_err(O[0].cpu().numpy(), m[0].cpu().numpy(), l[0].cpu().numpy(), Or.astype(np.float64),
                        mr.astype(np.float64), lr.astype(np.float64))
        comm.close()
        plan.close()
        ctx.close()
        q.put((rank, (res, e), None))
    except Exception as ex:
        q.put((rank, None, repr(ex)))


def test_rank_that_leaves_makes_the_bounded_exchange_time_out():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    old = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"          # no NVLink multicast objects bound while a rank leaves
    try:
        bound_ms = 3000
        q, procs = _spawn(_leaver, 2, bound_ms)
        got = {}
        try:
            for _ in range(2):
                rank, out, err = q.get(timeout=180)
                assert err is None, (rank, err)
                got[rank] = out
        finally:
            _join(procs)
    finally:
        if old is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = old
    assert got[1] == "left"
    (code, secs), e = got[0]
    # the deadline ran out (ETIMEOUT), or NCCL flagged the missing peer first (ENCCL): either way within the bound
    assert code in (pa.api.ETIMEOUT, pa.api.ENCCL), (code, secs)
    assert secs < bound_ms / 1000 + 15, secs
    assert e[0] <= TOL_REF and e[1] <= TOL_REF, e
