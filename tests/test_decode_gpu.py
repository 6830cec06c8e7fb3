"""Parity of the CUDA path (through the C ABI) with the oracle on identical seeded inputs.

Gates:
  * against the oracle's restatement of the reference's own arithmetic (f16 K/V/P, fp32 accumulation;
    scripts/sme/sme_attn.c:274-306): max |O - O_ref| / max |O_ref| <= 2e-3, |lse - lse_ref| <= 2e-3;
  * against the fp64 oracle with exact dequantisation (phone-attn/pa-tool.cpp:150-173): the reference's own gate,
    5e-3 on both (its f16 rounding of K, V and P alone costs ~2e-3 against exact arithmetic).
"""
import numpy as np
import pytest

import backburner_b200 as pa
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL_REF = 2e-3     # against the reference-arithmetic oracle
TOL_F64 = 5e-3     # against exact fp64 (pa-tool's gate)


def _dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _run(ctx, c, nk=None, segs_split=None):
    import torch
    sh = c["shape"]
    nk = c["K"].shape[0] if nk is None else nk
    shape = pa.shape_for(sh.hd, sh.nkv, sh.rows, sh.quant, sh.rs)
    K, V = _dev(c["K"]), _dev(c["V"])
    Qs = _dev(c["Qs"].view(np.int16)).view(torch.float16)
    bounds = segs_split or [0, nk]
    segs = [pa.Seg(K.data_ptr() + a * shape.rs, V.data_ptr() + a * shape.rs, b - a, 0)
            for a, b in zip(bounds[:-1], bounds[1:]) if b > a]
    O, m, l = pa.attn(ctx, shape, Qs, segs, 1)
    ctx.status()
    return O[0].cpu().numpy(), m[0].cpu().numpy(), l[0].cpu().numpy()


def _check(c, O, m, l, nk, tol_f64=TOL_F64):
    sh = c["shape"]
    Of, mf, lf = orc.partial_f64(sh, c["Qs"], c["K"], c["V"], nk)
    O3, m3, l3 = orc.partial_f32(sh, c["Qs"], c["K"], c["V"], nk)
    e64 = orc.rel_err(O, m, l, Of, mf, lf)
    e32 = orc.rel_err(O, m, l, O3.astype(np.float64), m3.astype(np.float64), l3.astype(np.float64))
    assert e32[0] <= TOL_REF and e32[1] <= TOL_REF, ("vs reference arithmetic", e32)
    assert e64[0] <= tol_f64 and e64[1] <= tol_f64, ("vs fp64", e64)
    # m itself is the row's exact maximum score, as sme_attn_partial returns it (scripts/sme/sme_attn.c:281,222-227),
    # on every kernel: not only a reference point that O and l are relative to
    valid = l3 > 0
    if valid.any():
        dm = np.abs(np.asarray(m, np.float64) - m3.astype(np.float64))[valid].max()
        assert dm <= TOL_REF, ("m vs reference arithmetic", dm)
    if nk == 0:
        assert np.all(l == 0) and np.all(np.isneginf(m)) and np.all(O == 0)
    return e32, e64


CASES = [
    # hd, nkv, rows, quant, nk                      what it covers
    (128, 8, 5, orc.Q8_0, 8192),                 # config 0 (1 token, GQA 5, 8,192 keys)
    (128, 8, 5, orc.Q4_0, 4096),                 # Q4_0 decode
    (128, 8, 80, orc.Q4_0, 2048),                # config 3 shape: 16 tokens x GQA 5, Q4_0
    (128, 8, 80, orc.Q8_0, 1000),
    (256, 4, 48, orc.Q8_0, 4096),                # pa-tool's wire geometry (HD 256, 48 rows, 4 KV heads)
    (256, 4, 48, orc.Q4_0, 2000),
    (256, 4, 6, orc.Q8_0, 1500),                 # one token of the wire geometry (rows packed)
    (128, 2, 10, orc.Q8_0, 333),
    (128, 8, 40, orc.Q8_0, 700),
    (128, 8, 16, orc.Q8_0, 64),
    (128, 8, 5, orc.F16, 4096),                  # f16 pages (store_f16 / is_q8 = 0), ldmatrix fragments
    (128, 8, 80, orc.F16, 1000),                 # f16 pages with many rows stay on the split-K kernel
    (256, 4, 48, orc.F16, 2000),                 # pa-tool's wire geometry with f16 pages
    (128, 2, 10, orc.F16, 333),
    (256, 4, 6, orc.F16, 77),
]


@pytest.mark.parametrize("which", [0, 1])   # the kernel the plan picks by shape; the split-K kernel forced
@pytest.mark.parametrize("hd,nkv,rows,quant,nk", CASES)
def test_decode_parity(ctx, hd, nkv, rows, quant, nk, which):
    c = orc.gen_case(1000 + hd + nkv + rows + nk + quant, hd, nkv, rows, nk, quant)
    ctx.set_kernel(which)
    try:
        O, m, l = _run(ctx, c)
    finally:
        ctx.set_kernel(0)
    _check(c, O, m, l, nk)


def _padded(c, pad):
    """The same case with `pad` unused bytes after each position's heads (rs > nkv * hb)."""
    sh = c["shape"]
    out = dict(c)
    for key in ("K", "V"):
        x = c[key]
        y = np.full((x.shape[0], x.shape[1] + pad), 0xEE, dtype=np.uint8)
        y[:, :x.shape[1]] = x
        out[key] = y
    out["shape"] = orc.shape(sh.hd, sh.nkv, sh.rows, sh.quant, rs=sh.rs + pad)
    return out


@pytest.mark.parametrize("hd,nkv,rows,quant,nk,pad", [
    (256, 16, 6, orc.Q8_0, 700, 0),      # 16 KV heads at hd 256: two head groups of 8 per position
    (128, 8, 5, orc.Q8_0, 999, 48),      # padded positions: the head group is not the whole row
    (128, 8, 5, orc.Q4_0, 300, 16),
    (128, 8, 5, orc.F16, 517, 32),       # f16: head groups of 4 and a padded row
])
def test_head_groups_and_padded_rows(ctx, hd, nkv, rows, quant, nk, pad):
    """Positions wider than one CTA's head group (or padded) are copied row by row instead of as contiguous pairs."""
    c = orc.gen_case(2000 + hd + nkv + nk + pad, hd, nkv, rows, nk, quant)
    if pad:
        c = _padded(c, pad)
    O, m, l = _run(ctx, c)
    _check(c, O, m, l, nk)


@pytest.mark.parametrize("nk", [0, 1, 2, 15, 16, 17, 31, 32, 33, 47, 63, 65, 100, 4097])
def test_ragged_key_counts(ctx, nk):
    c = orc.gen_case(77 + nk, 128, 8, 5, nk, orc.Q8_0)
    O, m, l = _run(ctx, c)
    _check(c, O, m, l, nk)


def test_student_t_values_and_large_scores(ctx):
    """config 4's heavy-tailed V, plus a large softmax scale (peaky scores) stress the LSE range."""
    c = orc.gen_case(4, 128, 8, 5, 3000, orc.Q8_0, student_t=True)
    O, m, l = _run(ctx, c)
    _check(c, O, m, l, 3000)
    # scale 0.5 instead of 1/sqrt(128): scores reach ~40, and the reference's f16 rounding of K alone moves them by
    # up to |s| * 2^-11 (~0.02): against exact fp64 the gate scales with the score range; against the reference's
    # own arithmetic it stays 2e-3
    c = orc.gen_case(5, 128, 8, 5, 3000, orc.Q8_0, scale=0.5)
    O, m, l = _run(ctx, c)
    _check(c, O, m, l, 3000, tol_f64=2e-2)


def test_segments_fold_like_one_run(ctx):
    """Keys split over several segments of one set (pages) give the same partial as one run."""
    c = orc.gen_case(9, 128, 8, 5, 5000, orc.Q8_0)
    O1, m1, l1 = _run(ctx, c)
    O2, m2, l2 = _run(ctx, c, segs_split=[0, 4096, 4100, 4100, 5000])
    e = orc.rel_err(O2, m2, l2, O1.astype(np.float64), m1.astype(np.float64), l1.astype(np.float64))
    assert e[0] < 1e-4 and e[1] < 1e-5, e
    _check(c, O2, m2, l2, 5000)


def test_many_sets_one_plan(ctx):
    """Several output sets (layers) with their own Q and keys in one plan, run twice."""
    import torch
    hd, nkv, rows = 128, 8, 5
    shape = pa.shape_for(hd, nkv, rows, pa.Q8_0)
    cases = [orc.gen_case(200 + i, hd, nkv, rows, nk, orc.Q8_0) for i, nk in enumerate([3000, 0, 129, 2048])]
    Ks = [_dev(c["K"]) for c in cases]
    Vs = [_dev(c["V"]) for c in cases]
    Qs = _dev(np.stack([c["Qs"] for c in cases]).view(np.int16)).view(torch.float16)
    segs = [pa.Seg(Ks[i].data_ptr(), Vs[i].data_ptr(), c["K"].shape[0], i) for i, c in enumerate(cases)]
    plan = pa.Plan(ctx, shape, len(cases), segs)
    O = torch.empty((len(cases), nkv, rows, hd), device="cuda")
    m = torch.empty((len(cases), nkv, rows), device="cuda")
    l = torch.empty_like(m)
    for _ in range(2):
        plan.run(Qs, O, m, l)
        ctx.status()
        for i, c in enumerate(cases):
            _check(c, O[i].cpu().numpy(), m[i].cpu().numpy(), l[i].cpu().numpy(), c["K"].shape[0])
    assert plan.launches == 2 and plan.scratch_bytes > 0
    plan.close()


def test_attn_partial_fp32_q(ctx):
    """sme_attn_partial's contract: fp32 unscaled Q, f16(q*scale) inside."""
    import torch
    c = orc.gen_case(31, 128, 8, 5, 2500, orc.Q8_0)
    shape = pa.shape_for(128, 8, 5, pa.Q8_0)
    O, m, l = pa.attn_partial(ctx, shape, _dev(c["Q"]), c["scale"], _dev(c["K"]), _dev(c["V"]), 2500)
    _check(c, O.cpu().numpy(), m.cpu().numpy(), l.cpu().numpy(), 2500)


def test_scale_q_bit_exact(ctx):
    import torch
    rng = np.random.default_rng(0)
    Q = (rng.standard_normal(100000) * 50).astype(np.float32)
    got = pa.scale_q(ctx, _dev(Q), 0.0883883).cpu().numpy().view(np.uint16)
    assert np.array_equal(got, orc.scale_q(Q, 0.0883883))


@pytest.mark.parametrize("hd", [128, 256])
def test_merge_kernel_matches_oracle(ctx, hd):
    import torch
    rng = np.random.default_rng(hd)
    n, rows = 5, 37
    Op = rng.standard_normal((n, rows, hd)).astype(np.float32)
    mp = (rng.standard_normal((n, rows)) * 4).astype(np.float32)
    lp = (np.abs(rng.standard_normal((n, rows))) + 0.1).astype(np.float32)
    lp[1, :5] = 0.0
    mp[1, :5] = -np.inf          # empty parts are skipped
    lp[:, 7] = 0.0
    mp[:, 7] = -np.inf           # a row with no keys anywhere
    O, m, l = pa.merge(ctx, hd, _dev(Op), _dev(mp), _dev(lp))
    torch.cuda.synchronize()
    Or, mr, lr = orc.merge_slots(Op, mp, lp)
    np.testing.assert_allclose(O.cpu().numpy(), Or, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(l.cpu().numpy(), lr, rtol=2e-5)
    assert np.isneginf(m.cpu().numpy()[7]) and l.cpu().numpy()[7] == 0
    # fold: (O, m, l) already holds a partial (merge_partial / pa_merge_big's fold bit)
    O0 = rng.standard_normal((rows, hd)).astype(np.float32)
    m0 = rng.standard_normal(rows).astype(np.float32)
    l0 = (np.abs(rng.standard_normal(rows)) + 0.1).astype(np.float32)
    out = (_dev(O0), _dev(m0), _dev(l0))
    pa.merge(ctx, hd, _dev(Op[:1]), _dev(mp[:1]), _dev(lp[:1]), out=out, fold=True)
    torch.cuda.synchronize()
    Oc, mc, lc = O0.copy(), m0.copy(), l0.copy()
    orc.merge_partial(Oc, mc, lc, Op[0], mp[0], lp[0])
    np.testing.assert_allclose(out[0].cpu().numpy(), Oc, rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(out[2].cpu().numpy(), lc, rtol=2e-5)


@pytest.mark.parametrize("hd,n,rows", [(128, 100, 24), (256, 257, 6), (128, 9, 40), (256, 33, 3000)])
def test_merge_many_parts_matches_oracle(ctx, hd, n, rows):
    """Few rows with many parts (the merge deals a row's parts out to 8 warps) and many rows (one warp per row): empty
    parts (l = 0) whose O holds NaN must add nothing, as merge_partial skips them; the fold takes one more part."""
    import torch
    rng = np.random.default_rng(hd + n + rows)
    Op = rng.standard_normal((n, rows, hd)).astype(np.float32)
    mp = (rng.standard_normal((n, rows)) * 4).astype(np.float32)
    lp = (np.abs(rng.standard_normal((n, rows))) + 0.1).astype(np.float32)
    empty = rng.random((n, rows)) < 0.2
    lp[empty] = 0.0
    mp[empty] = -np.inf
    Op[empty] = np.nan
    lp[:, 1] = 0.0
    mp[:, 1] = -np.inf           # a row with no keys anywhere
    Op[:, 1] = np.nan
    O, m, l = pa.merge(ctx, hd, _dev(Op), _dev(mp), _dev(lp))
    torch.cuda.synchronize()
    Or, mr, lr = orc.merge_slots(np.where(np.isnan(Op), 0, Op), mp, lp)
    np.testing.assert_allclose(O.cpu().numpy(), Or, rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(l.cpu().numpy(), lr, rtol=3e-5)
    np.testing.assert_array_equal(m.cpu().numpy()[lr > 0], mr[lr > 0])
    assert np.isneginf(m.cpu().numpy()[1]) and l.cpu().numpy()[1] == 0 and np.all(O.cpu().numpy()[1] == 0)
    O0 = rng.standard_normal((rows, hd)).astype(np.float32)
    m0 = rng.standard_normal(rows).astype(np.float32)
    l0 = (np.abs(rng.standard_normal(rows)) + 0.1).astype(np.float32)
    out = (_dev(O0), _dev(m0), _dev(l0))
    pa.merge(ctx, hd, _dev(Op), _dev(mp), _dev(lp), out=out, fold=True)
    torch.cuda.synchronize()
    Oc, mc, lc = O0.copy(), m0.copy(), l0.copy()
    Om = np.where(np.isnan(Op), 0, Op)
    for c in range(n):
        orc.merge_partial(Oc, mc, lc, Om[c], mp[c], lp[c])
    np.testing.assert_allclose(out[0].cpu().numpy(), Oc, rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(out[2].cpu().numpy(), lc, rtol=3e-5)


def test_normalize_matches_attn_core(ctx):
    import torch
    rng = np.random.default_rng(2)
    rows, hd = 50, 128
    O = rng.standard_normal((rows, hd)).astype(np.float32) * 3
    m = rng.standard_normal(rows).astype(np.float32)
    l = (np.abs(rng.standard_normal(rows)) + 0.2).astype(np.float32)
    l[3] = 0.0
    Oh, lse = pa.normalize(ctx, hd, _dev(O), _dev(m), _dev(l))
    torch.cuda.synchronize()
    Ohr, lser = orc.normalize(O, m, l)
    assert np.array_equal(Oh.cpu().numpy().view(np.uint16), Ohr)
    np.testing.assert_allclose(lse.cpu().numpy(), lser, rtol=1e-6, atol=1e-6)


def test_fold_reply_matches_oracle(ctx):
    """pa_cuda_fold_reply: the engine's partial over the offloaded keys goes out normalised (ATTN's reply: f16 O/l,
    lse) and is folded into the host's own unnormalised partial as O_unnorm = O, l = 1, m = lse
    (phone-attn.h:18-20). Checked against the oracle's fold of the same reply bits, and the folded result against
    the oracle over all keys at the 2e-3 gate; rows with an empty reply or an empty host partial included."""
    import torch
    c = orc.gen_case(4321, 128, 8, 40, 6000, orc.Q8_0)
    sh = c["shape"]
    na = 5000
    shape = pa.shape_for(128, 8, 40, pa.Q8_0)
    K, V = _dev(c["K"][:na]), _dev(c["V"][:na])
    Qs = _dev(c["Qs"].view(np.int16)).view(torch.float16)
    O, m, l = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), na, 0)])
    Oh, lse = pa.normalize(ctx, 128, O.reshape(-1, 128), m.reshape(-1), l.reshape(-1))
    lse[7] = -float("inf")                                    # an empty reply row
    OB, mB, lB = orc.partial_f32(sh, c["Qs"], c["K"][na:], c["V"][na:], 6000 - na)
    lB = lB.copy()
    lB.reshape(-1)[11] = 0.0                                  # an empty host row
    Od, md, ld = _dev(OB.reshape(-1, 128)), _dev(mB.reshape(-1)), _dev(lB.reshape(-1))
    pa.fold_reply(ctx, 128, Oh, lse, Od, md, ld)
    ctx.status()
    Oh_h, lse_h = Oh.cpu().numpy().view(np.uint16), lse.cpu().numpy()
    Or, mr, lr = OB.reshape(-1, 128).copy(), mB.reshape(-1).copy(), lB.reshape(-1).copy()
    orc.fold_reply(Or, mr, lr, Oh_h, lse_h)
    np.testing.assert_allclose(Od.cpu().numpy(), Or, rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(md.cpu().numpy(), mr, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(ld.cpu().numpy(), lr, rtol=2e-5)
    # the folded partial against the oracle over all keys (rows without an empty side)
    Oa, ma, la = orc.partial_f32(sh, c["Qs"], c["K"], c["V"], 6000)
    keep = np.ones(8 * 40, bool)
    keep[[7, 11]] = False
    got = (Od.cpu().numpy()[keep], md.cpu().numpy()[keep], ld.cpu().numpy()[keep])
    e = orc.rel_err(*got, Oa.reshape(-1, 128)[keep].astype(np.float64), ma.reshape(-1)[keep].astype(np.float64),
                    la.reshape(-1)[keep].astype(np.float64))
    assert e[0] <= TOL_REF and e[1] <= TOL_REF, e


@pytest.mark.parametrize("quant,ntok,ng", [(orc.Q8_0, 8, 1), (orc.Q8_0, 1, 1), (orc.Q8_0, 3, 1), (orc.Q4_0, 8, 1),
                                           (orc.Q8_0, 8, 3)])
def test_engine_pages_begin_end(ctx, quant, ntok, ng):
    """pa::engine contract: engine pages written by the host (as pa::server's APPEND does), begin() with f16(q*scale)
    in the wire layout [ng][nkv][48][256], end() unnormalised O/m/l; rows t >= ntok come back empty."""
    hd, nkv, NR, PAGE = 256, 4, 48, 4096
    nk = 6000
    c = orc.gen_case(55 + ntok + quant, hd, nkv, NR * ng, nk, quant)
    # wire layout: per group g, [nkv][48][hd]; rows t >= ntok zeroed (pa-tool.cpp:141)
    Qs = c["Qs"].reshape(nkv, ng, NR, hd).transpose(1, 0, 2, 3).copy()
    if ng == 1 and ntok < 8:
        Qs[:, :, (np.arange(NR) % 8) >= ntok, :] = 0
    shape = pa.shape_for(hd, nkv, NR, quant)
    eng = pa.Engine(ctx)
    pages, nkeys = [], []
    for p0 in range(0, nk, PAGE):
        n = min(PAGE, nk - p0)
        pg = eng.alloc_page(PAGE * shape.rs)
        eng.page_view(pg, n * shape.rs, "k")[:] = c["K"][p0:p0 + n].ravel()
        eng.page_view(pg, n * shape.rs, "v")[:] = c["V"][p0:p0 + n].ravel()
        pages.append(pg)
        nkeys.append(n)
    O = np.empty((ng, nkv * NR, hd), np.float32)
    m = np.empty((ng, nkv * NR), np.float32)
    l = np.empty_like(m)
    for _ in range(2):
        eng.begin(pages, nkeys, Qs, shape, ng, ntok)
        assert eng.end(O, m, l) >= 0
    for g in range(ng):
        Qg = Qs[g].reshape(nkv, NR, hd)
        sh = orc.shape(hd, nkv, NR, quant)
        Of, mf, lf = orc.partial_f64(sh, Qg, c["K"], c["V"], nk)
        real = (np.arange(NR) % 8) < (ntok if ng == 1 else 8)
        Og, mg, lg = O[g].reshape(nkv, NR, hd), m[g].reshape(nkv, NR), l[g].reshape(nkv, NR)
        e = orc.rel_err(Og[:, real], mg[:, real], lg[:, real], Of[:, real], mf[:, real], lf[:, real])
        assert e[0] <= TOL_F64 and e[1] <= TOL_F64, e
        if not real.all():
            assert np.all(lg[:, ~real] == 0) and np.all(np.isneginf(mg[:, ~real]))
    for pg in pages:
        eng.free_page(pg)


@pytest.mark.parametrize("ntok", [1, 8])
def test_engine_arm_replays_the_call_as_a_graph(ctx, ntok):
    """engine::arm (phone-attn/phone-attn.h:179-182): after arm(), a begin with the same pages, key counts and tokens
    replays a CUDA graph of the whole call and returns exactly what the plain path returned; the graph stays with the
    call's cached plan, so later calls of that shape replay it too, each reading its own Q; a call of another shape runs
    the plain path."""
    hd, nkv, NR, PAGE, quant = 256, 4, 48, 4096, orc.Q8_0
    nk = 9000
    c = orc.gen_case(71 + ntok, hd, nkv, NR, nk, quant)
    c2 = orc.gen_case(72 + ntok, hd, nkv, NR, nk, quant)
    def wire(cc):
        q = cc["Qs"].reshape(nkv, 1, NR, hd).transpose(1, 0, 2, 3).copy()
        q[:, :, (np.arange(NR) % 8) >= ntok, :] = 0
        return q
    Qa, Qb = wire(c), wire(c2)
    shape = pa.shape_for(hd, nkv, NR, quant)
    sh = orc.shape(hd, nkv, NR, quant)
    real = (np.arange(NR) % 8) < ntok
    eng = pa.Engine(ctx)
    pages, nkeys = [], []
    for p0 in range(0, nk, PAGE):
        n = min(PAGE, nk - p0)
        pg = eng.alloc_page(PAGE * shape.rs)
        eng.page_view(pg, n * shape.rs, "k")[:] = c["K"][p0:p0 + n].ravel()
        eng.page_view(pg, n * shape.rs, "v")[:] = c["V"][p0:p0 + n].ravel()
        pages.append(pg)
        nkeys.append(n)
    out = lambda: (np.empty((1, nkv * NR, hd), np.float32), np.empty((1, nkv * NR), np.float32),
                   np.empty((1, nkv * NR), np.float32))
    def check(res, Q, n):
        Of, mf, lf = orc.partial_f64(sh, Q[0].reshape(nkv, NR, hd), c["K"][:n], c["V"][:n], n)
        O, m, l = res
        e = orc.rel_err(O[0].reshape(nkv, NR, hd)[:, real], m[0].reshape(nkv, NR)[:, real], l[0].reshape(nkv, NR)[:, real],
                        Of[:, real], mf[:, real], lf[:, real])
        assert e[0] <= TOL_F64 and e[1] <= TOL_F64, e
    g0 = eng.graph_calls
    r1 = out()
    eng.begin(pages, nkeys, Qa, shape, 1, ntok)
    assert eng.end(*r1) >= 0
    assert eng.graph_calls == g0                      # not armed yet: the plain path
    eng.arm(pages, nkeys, shape, ntok)
    r2 = out()
    eng.begin(pages, nkeys, Qa, shape, 1, ntok)
    assert eng.end(*r2) >= 0
    assert eng.graph_calls == g0 + 1
    assert all(np.array_equal(a, b) for a, b in zip(r1, r2))
    r3 = out()                                       # another shape (the first page only), never armed: plain path
    eng.begin(pages[:1], nkeys[:1], Qa, shape, 1, ntok)
    assert eng.end(*r3) >= 0
    assert eng.graph_calls == g0 + 1
    check(r3, Qa, nkeys[0])
    r4 = out()                                       # the armed shape again, with another Q: replayed, new Q read
    eng.begin(pages, nkeys, Qb, shape, 1, ntok)
    assert eng.end(*r4) >= 0
    assert eng.graph_calls == g0 + 2
    check(r4, Qb, nk)
    for pg in pages:
        eng.free_page(pg)


def test_bounded_wait_reports_and_context_recovers(ctx):
    """Failure detection without a GPU fault: with the stall hook on, the consumer warps wait on a barrier that nothing
    completes; after the 1 ms limit the kernel records the timeout and returns (no trap), the host reads ETIMEOUT,
    and the next call on the same context is correct."""
    c = orc.gen_case(3, 128, 8, 5, 4096, orc.Q8_0)
    ctx.set_timeout_ns(1_000_000)
    ctx.set_stall_test(True)
    try:
        with pytest.raises(pa.PaCudaError) as ei:
            _run(ctx, c)
        assert ei.value.code == -4
    finally:
        ctx.set_stall_test(False)
        ctx.set_timeout_ns(2_000_000_000)
    O, m, l = _run(ctx, c)
    _check(c, O, m, l, 4096)


def test_full_layer_size_against_fp64(ctx):
    """One full layer of config 1 (131,072 Q8_0 keys, 8 KV heads, GQA 5) against the fp64 oracle."""
    nk = 131072
    c = orc.gen_case(2024, 128, 8, 5, nk, orc.Q8_0)
    O, m, l = _run(ctx, c)
    sh = c["shape"]
    Of, mf, lf = orc.partial_f64(sh, c["Qs"], c["K"], c["V"], nk)
    e = orc.rel_err(O, m, l, Of, mf, lf)
    assert e[0] <= TOL_F64 and e[1] <= TOL_F64, e
