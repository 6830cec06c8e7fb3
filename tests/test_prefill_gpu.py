"""Parity of the tcgen05/TMEM kernel (many query rows per KV head: prefill, ATTN_BIG, long verify batches) with the
oracle on identical seeded inputs, and with the split-K mma.sync kernel on the same call. Tolerances as in
test_decode_gpu.py: 2e-3 against the reference-arithmetic oracle, 5e-3 (pa-tool's gate) against exact fp64."""
import numpy as np
import pytest

import backburner_b200 as pa
from oracle import oracle as orc

from test_decode_gpu import TOL_F64, TOL_REF, _check, _dev

pytestmark = pytest.mark.gpu


def _run_kernel(ctx, c, which, n_sets=1, cases=None):
    import torch
    ctx.set_kernel(which)
    try:
        sh = c["shape"]
        shape = pa.shape_for(sh.hd, sh.nkv, sh.rows, sh.quant)
        K, V = _dev(c["K"]), _dev(c["V"])
        Qs = _dev(c["Qs"].view(np.int16)).view(torch.float16)
        nk = c["K"].shape[0]
        O, m, l = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), nk, 0)], 1)
        ctx.status()
        return O[0].cpu().numpy(), m[0].cpu().numpy(), l[0].cpu().numpy()
    finally:
        ctx.set_kernel(0)


@pytest.mark.parametrize("rows,nk,quant", [
    (64, 1024, orc.Q8_0), (80, 2048, orc.Q4_0), (80, 1000, orc.Q8_0), (128, 4096, orc.Q8_0), (129, 700, orc.Q8_0),
    (256, 2048, orc.Q8_0), (300, 1500, orc.Q4_0), (640, 4096, orc.Q8_0), (5, 333, orc.Q8_0), (48, 64, orc.Q8_0),
    (256, 1, orc.Q8_0), (200, 63, orc.Q4_0), (257, 65, orc.Q8_0)])
def test_tcgen05_kernel_parity(ctx, rows, nk, quant):
    c = orc.gen_case(3000 + rows + nk + quant, 128, 8, rows, nk, quant)
    O, m, l = _run_kernel(ctx, c, 2)
    _check(c, O, m, l, nk)


# the CTA-pair instance (kernel 3): 256-row pair tiles, NT = 1 up to 256 rows and 2 above; ragged rows and keys
@pytest.mark.parametrize("rows,nk,quant", [
    (512, 4096, orc.Q8_0), (640, 4096, orc.Q8_0), (300, 1500, orc.Q4_0), (129, 700, orc.Q8_0), (257, 65, orc.Q8_0),
    (256, 1, orc.Q8_0), (200, 63, orc.Q4_0), (1024, 2048, orc.Q4_0), (5, 333, orc.Q8_0), (768, 97, orc.Q8_0)])
def test_tcgen05_pair_kernel_parity(ctx, rows, nk, quant):
    c = orc.gen_case(5000 + rows + nk + quant, 128, 8, rows, nk, quant)
    O, m, l = _run_kernel(ctx, c, 3)
    _check(c, O, m, l, nk)


# head dim 256 (the reference server's wire geometry: HD 256, 48 rows per group, phone-attn.h:79-80) on the pair
# kernel (the default above 128 rows per KV head; forced here for every size): ATTN_BIG groups (rows = 48 ng), an
# 8-token ATTN (48 rows), ragged keys, Q4_0
@pytest.mark.parametrize("rows,nk,quant", [
    (96, 2048, orc.Q8_0), (144, 4096, orc.Q8_0), (256, 1500, orc.Q4_0), (512, 777, orc.Q8_0), (300, 65, orc.Q8_0),
    (64, 1, orc.Q4_0), (768, 3000, orc.Q8_0), (48, 2500, orc.Q8_0), (32, 999, orc.Q4_0)])
def test_tcgen05_pair_kernel_hd256_parity(ctx, rows, nk, quant):
    c = orc.gen_case(7000 + rows + nk + quant, 256, 8, rows, nk, quant)
    O, m, l = _run_kernel(ctx, c, 3)
    _check(c, O, m, l, nk)


# head dim 256 on the single-CTA kernel with one 128-row tile (the default from 9 to 128 rows per KV head): an 8-token
# ATTN (48 rows), a 2-token one (12), two groups (96), a full tile, ragged keys, Q4_0, and more rows than one tile
# (forced: several tiles per head as separate CTAs)
@pytest.mark.parametrize("rows,nk,quant", [
    (48, 2500, orc.Q8_0), (12, 3000, orc.Q8_0), (96, 2048, orc.Q8_0), (128, 4096, orc.Q8_0), (32, 999, orc.Q4_0),
    (64, 1, orc.Q4_0), (80, 65, orc.Q8_0), (200, 777, orc.Q8_0)])
def test_tcgen05_kernel_hd256_parity(ctx, rows, nk, quant):
    c = orc.gen_case(7500 + rows + nk + quant, 256, 8, rows, nk, quant)
    O, m, l = _run_kernel(ctx, c, 0 if rows <= 128 else 2)
    _check(c, O, m, l, nk)


def test_hd256_plans_pick_their_kernels(ctx):
    import torch
    for rows, want in [(8, "pa::dec::decode_kernel<256,1,8>"), (12, "pa::pre::prefill_kernel<1,1,256>"),
                       (48, "pa::pre::prefill_kernel<1,1,256>"),
                       (128, "pa::pre::prefill_kernel<1,1,256>"), (144, "pa::pre::prefill_pair_kernel<1,1,256>")]:
        shape = pa.shape_for(256, 8, rows, pa.Q8_0)
        K = torch.zeros((128, shape.rs), dtype=torch.uint8, device="cuda")
        plan = pa.Plan(ctx, shape, 1, [pa.Seg(K.data_ptr(), K.data_ptr(), 128, 0)])
        assert plan.kernel == want
        plan.close()


@pytest.mark.parametrize("hd,rows,nk", [(128, 80, 3000), (128, 256, 2000), (256, 192, 2500), (256, 48, 3000)])
def test_tcgen05_matches_split_k_kernel(ctx, hd, rows, nk):
    c = orc.gen_case(77 + rows, hd, 8, rows, nk, orc.Q8_0)
    O1, m1, l1 = _run_kernel(ctx, c, 1)
    for which in (2, 3):
        O2, m2, l2 = _run_kernel(ctx, c, which)
        e = orc.rel_err(O2, m2, l2, O1.astype(np.float64), m1.astype(np.float64), l1.astype(np.float64))
        assert e[0] <= 1e-3 and e[1] <= 1e-3, (which, e)


@pytest.mark.parametrize("which,rows", [(2, 160), (3, 160), (3, 600)])
def test_tcgen05_many_sets_and_split_keys(ctx, which, rows):
    """Several layers (output sets) in one plan, each split into several key chunks (jobs), run twice."""
    import torch
    hd, nkv = 128, 8
    ctx.set_kernel(which)
    try:
        shape = pa.shape_for(hd, nkv, rows, pa.Q8_0)
        cases = [orc.gen_case(900 + i, hd, nkv, rows, nk, orc.Q8_0) for i, nk in enumerate([5000, 64, 2100])]
        Ks = [_dev(c["K"]) for c in cases]
        Vs = [_dev(c["V"]) for c in cases]
        Qs = _dev(np.stack([c["Qs"] for c in cases]).view(np.int16)).view(torch.float16)
        segs = [pa.Seg(Ks[i].data_ptr(), Vs[i].data_ptr(), c["K"].shape[0], i) for i, c in enumerate(cases)]
        plan = pa.Plan(ctx, shape, len(cases), segs, chunk_keys=1024)
        O = torch.empty((len(cases), nkv, rows, hd), device="cuda")
        m = torch.empty((len(cases), nkv, rows), device="cuda")
        l = torch.empty_like(m)
        for _ in range(2):
            plan.run(Qs, O, m, l)
            ctx.status()
            for i, c in enumerate(cases):
                _check(c, O[i].cpu().numpy(), m[i].cpu().numpy(), l[i].cpu().numpy(), c["K"].shape[0])
        plan.close()
    finally:
        ctx.set_kernel(0)


@pytest.mark.parametrize("which", [2, 3])
def test_tcgen05_student_t_values(ctx, which):
    c = orc.gen_case(44, 128, 8, 256, 3000, orc.Q8_0, student_t=True)
    O, m, l = _run_kernel(ctx, c, which)
    _check(c, O, m, l, 3000)


@pytest.mark.parametrize("which,hd,rows", [(2, 128, 256), (3, 128, 512), (3, 256, 96), (2, 256, 96)])
def test_tcgen05_bounded_wait_reports_and_context_recovers(ctx, which, hd, rows):
    """Failure detection without a GPU fault, on the tcgen05 kernels (single CTA and CTA pair, hd 128 and 256): with the
    stall hook on, the softmax warps wait on a barrier that nothing completes; after the 1 ms limit the kernel records
    the timeout, every role of both CTAs of a pair unwinds through its bounded waits, TMEM is freed, the host reads
    ETIMEOUT, and the next call on the same context is correct."""
    c = orc.gen_case(55 + hd + rows, hd, 8, rows, 2048, orc.Q8_0)
    ctx.set_timeout_ns(1_000_000)
    ctx.set_stall_test(True)
    try:
        with pytest.raises(pa.PaCudaError) as ei:
            _run_kernel(ctx, c, which)
        assert ei.value.code == -4
    finally:
        ctx.set_stall_test(False)
        ctx.set_timeout_ns(2_000_000_000)
    O, m, l = _run_kernel(ctx, c, which)
    _check(c, O, m, l, 2048)
