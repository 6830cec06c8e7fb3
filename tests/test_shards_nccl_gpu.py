"""pa_cuda_shard_attn_allgather_merge: position shards over NCCL in one call (one process per GPU; each rank's plan covers
its contiguous range of positions; one ncclAllGather exchanges the packed (O, m, l); every rank folds all of them).
A communicator of one rank must give exactly what the plan alone gives; two ranks on two GPUs must agree with each
other and with the oracle over all positions (2e-3, as the other parity tests). The two-rank test needs two GPUs."""
import numpy as np
import pytest

import backburner_b200 as pa
from oracle import oracle as orc

from test_decode_gpu import TOL_REF

pytestmark = pytest.mark.gpu


def test_one_rank_equals_the_plan(ctx):
    import torch
    c = orc.gen_case(61, 128, 8, 5, 3000, orc.Q8_0)
    shape = pa.shape_for(128, 8, 5, pa.Q8_0)
    K, V = torch.from_numpy(c["K"]).cuda(), torch.from_numpy(c["V"]).cuda()
    Qs = torch.from_numpy(c["Qs"].view(np.int16)).cuda().view(torch.float16)
    plan = pa.Plan(ctx, shape, 1, [pa.Seg(K.data_ptr(), V.data_ptr(), 3000, 0)])
    O1 = torch.empty((1, 8, 5, 128), device="cuda")
    m1 = torch.empty((1, 8, 5), device="cuda")
    l1 = torch.empty_like(m1)
    plan.run(Qs, O1, m1, l1)
    comm = pa.NcclComm(ctx, pa.nccl_unique_id(), 0, 1)
    try:
        for _ in range(2):
            O2, m2, l2 = torch.empty_like(O1), torch.empty_like(m1), torch.empty_like(l1)
            pa.shard_attn_allgather_merge(plan, Qs, comm, O2, m2, l2)
            ctx.status()
            np.testing.assert_allclose(O2.cpu().numpy(), O1.cpu().numpy(), rtol=1e-6, atol=1e-7)
            np.testing.assert_allclose(m2.cpu().numpy(), m1.cpu().numpy(), rtol=1e-6)
            np.testing.assert_allclose(l2.cpu().numpy(), l1.cpu().numpy(), rtol=1e-6)
    finally:
        comm.close()
        plan.close()


def _rank(rank, world, uid, q):
    try:
        import torch
        import backburner_b200 as pa2
        torch.cuda.set_device(rank)
        ctx = pa2.Context(rank)
        c = orc.gen_case(62, 128, 8, 5, 5000, orc.Q8_0)           # the same seeded case on every rank
        a, b = rank * 5000 // world, (rank + 1) * 5000 // world
        shape = pa2.shape_for(128, 8, 5, pa2.Q8_0)
        dev = torch.device("cuda", rank)
        K = torch.from_numpy(np.ascontiguousarray(c["K"][a:b])).to(dev)
        V = torch.from_numpy(np.ascontiguousarray(c["V"][a:b])).to(dev)
        Qs = torch.from_numpy(c["Qs"].view(np.int16)).to(dev).view(torch.float16)
        plan = pa2.Plan(ctx, shape, 1, [pa2.Seg(K.data_ptr(), V.data_ptr(), b - a, 0)])
        comm = pa2.NcclComm(ctx, uid, rank, world)
        O = torch.empty((1, 8, 5, 128), device=dev)
        m = torch.empty((1, 8, 5), device=dev)
        l = torch.empty_like(m)
        out = []
        for _ in range(2):
            pa2.shard_attn_allgather_merge(plan, Qs, comm, O, m, l)
            ctx.status()
            out.append((O.cpu().numpy(), m.cpu().numpy(), l.cpu().numpy()))
        comm.close()
        plan.close()
        ctx.close()
        q.put((rank, out, None))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def test_two_ranks_on_two_gpus_match_the_oracle():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    uid = pa.nccl_unique_id()
    ctxm = mp.get_context("spawn")
    q = ctxm.Queue()
    procs = [ctxm.Process(target=_rank, args=(r, 2, uid, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    try:
        for _ in range(2):
            rank, out, err = q.get(timeout=180)
            assert err is None, (rank, err)
            got[rank] = out
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    c = orc.gen_case(62, 128, 8, 5, 5000, orc.Q8_0)
    Or, mr, lr = orc.partial_f32(c["shape"], c["Qs"], c["K"], c["V"], 5000)
    for rank in (0, 1):
        for O, m, l in got[rank]:
            e = orc.rel_err(O[0], m[0], l[0], Or.astype(np.float64), mr.astype(np.float64), lr.astype(np.float64))
            assert e[0] <= TOL_REF and e[1] <= TOL_REF, (rank, e)
    np.testing.assert_array_equal(got[0][0][0], got[1][0][0])      # the fold is the same on every rank
