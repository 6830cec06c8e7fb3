"""The int8-domain QK (scripts/sme/sme_attn.c:465-508: sme_qk_i8blk's per-32-block int32 dot products of int8 Q and
Q8_0 K, combined by i8_combine as s = sum_b float(T_b) * dq_b * dk_b) on the split-K kernel, opt-in through
pa_cuda_set_qk_domain, against the oracle's restatement of the same arithmetic (orc_partial_f32_i8q).

Gates: the scores are exact integer block products combined in the oracle's order, so the row maxima m match it bit for
bit; O/l and lse within 2e-3 (the softmax's exp2 and the f16 rounding of P differ in the last bits)."""
import numpy as np
import pytest

import backburner_b200 as pa
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(ctx, c, bounds):
    import torch
    sh = c["shape"]
    shape = pa.shape_for(sh.hd, sh.nkv, sh.rows, sh.quant, sh.rs)
    K, V = _dev(c["K"]), _dev(c["V"])
    Qs = _dev(c["Qs"].view(np.int16)).view(torch.float16)
    segs = [pa.Seg(K.data_ptr() + a * shape.rs, V.data_ptr() + a * shape.rs, b - a, 0)
            for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
    plan = pa.Plan(ctx, shape, 1, segs)
    name = plan.kernel
    plan.close()
    O, m, l = pa.attn(ctx, shape, Qs, segs, 1)
    ctx.status()
    return name, O[0].cpu().numpy(), m[0].cpu().numpy(), l[0].cpu().numpy()


CASES = [
    # hd, nkv, rows, nk, split                    what it covers
    (128, 8, 5, 8192, None),                     # config 0's shape (1 token, GQA 5)
    (128, 8, 80, 1000, None),                    # 16 tokens x GQA 5: many rows stay on the split-K kernel
    (128, 2, 10, 333, None),                     # a ragged tail stage
    (128, 8, 16, 64, [0, 17, 64]),               # two segments, the first of odd length
    (256, 4, 48, 4096, None),                    # pa-tool's wire geometry
    (256, 4, 6, 1500, [0, 700, 1500]),
    (256, 8, 5, 2000, None),                     # hd 256 with 8 KV heads per CTA
    (128, 8, 5, 0, None),                        # no keys: the empty partial
]


@pytest.mark.parametrize("hd,nkv,rows,nk,split", CASES)
def test_int8_domain_qk_matches_oracle(ctx, hd, nkv, rows, nk, split):
    c = orc.gen_case(4000 + hd + nkv + rows + nk, hd, nkv, rows, nk, orc.Q8_0)
    ctx.set_qk_domain(pa.QK_INT8)
    try:
        name, O, m, l = _run(ctx, c, split or [0, nk])
    finally:
        ctx.set_qk_domain(pa.QK_F16)
    assert ",3," in name and name.startswith("pa::dec::decode_kernel<"), name
    if nk == 0:
        assert np.all(l == 0) and np.all(np.isneginf(m)) and np.all(O == 0)
        return
    O2, m2, l2 = orc.partial_f32_i8q(c["shape"], c["Qs"], c["K"], c["V"], nk)
    e = orc.rel_err(O, m, l, O2.astype(np.float64), m2.astype(np.float64), l2.astype(np.float64))
    assert e[0] <= TOL and e[1] <= TOL, e
    valid = l2 > 0
    assert valid.all()
    assert np.array_equal(m[valid], m2[valid]), np.abs(m - m2).max()
    # and it is the int8 arithmetic, not the f16 one: the f16-domain oracle's maxima differ
    O1, m1, l1 = orc.partial_f32(c["shape"], c["Qs"], c["K"], c["V"], nk)
    assert not np.array_equal(m1, m2)


def test_int8_domain_qk_refuses_other_rows_and_kernels(ctx):
    import torch
    ctx.set_qk_domain(pa.QK_INT8)
    try:
        for quant, which in [(pa.Q4_0, 0), (pa.F16, 0), (pa.Q8_0, 2), (pa.Q8_0, 3)]:
            shape = pa.shape_for(128, 8, 5, quant)
            K = torch.zeros((64, shape.rs), dtype=torch.uint8, device="cuda")
            ctx.set_kernel(which)
            with pytest.raises(pa.PaCudaError) as ei:
                pa.Plan(ctx, shape, 1, [pa.Seg(K.data_ptr(), K.data_ptr(), 64, 0)])
            assert ei.value.code == -5 and "int8-domain" in str(ei.value)
        # Q8_0 rows with many query rows per KV head take the split-K kernel, not the tcgen05 ones
        ctx.set_kernel(0)
        shape = pa.shape_for(128, 8, 160, pa.Q8_0)
        K = torch.zeros((64, shape.rs), dtype=torch.uint8, device="cuda")
        plan = pa.Plan(ctx, shape, 1, [pa.Seg(K.data_ptr(), K.data_ptr(), 64, 0)])
        assert plan.kernel == "pa::dec::decode_kernel<128,3,8>"
        plan.close()
    finally:
        ctx.set_kernel(0)
        ctx.set_qk_domain(pa.QK_F16)
