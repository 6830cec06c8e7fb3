"""The allocation-free entry point (pa_cuda_attn_noalloc), called through the C ABI.

Some callers cannot allocate device memory themselves: a host runtime that owns all device memory in its own pool, or
an inference server that has reserved the GPU up front, cannot create a context or a plan, because both allocate
scratch. pa_cuda_attn_noalloc runs the same split-K kernel and merge on a fixed device array compiled into the library.
Here two calls in a row (different inputs, so the second cannot pass on the first call's leftovers) must match the
oracle (the reference's own arithmetic, and exact fp64 at pa-tool's gate) and the allocating entry point, pa_cuda_attn,
within the tolerance of the other parity tests; a third case is sized so that its chunk partials nearly fill the fixed
array (3 slots), the path where the chunk size is raised past the usual cap. The file is named to be collected last and
needs nothing from the other test files, so it passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest

import backburner_b200 as pa
from backburner_b200 import api
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL = 2e-3       # the parity tolerance of the other GPU tests (against the reference-arithmetic oracle)
TOL_F64 = 5e-3   # against exact fp64 (pa-tool's gate)


def _noalloc(shape, Qs, K, V, nk, O, m, l):
    why = ctypes.c_char_p()
    sh = shape.c()
    rc = pa.lib().pa_cuda_attn_noalloc(ctypes.byref(sh), Qs.data_ptr(), K.data_ptr(), V.data_ptr(), nk, O.data_ptr(),
                                       m.data_ptr(), l.data_ptr(), api._stream_ptr(None), ctypes.byref(why))
    return rc, (why.value or b"").decode()


def _vs_oracle(c, O, m, l, nk, rows_idx=None):
    """(O, m, l) of the call against the oracle on the rows rows_idx (all rows by default): rows are independent, so
    a sample of rows is an exact check of those rows."""
    sh = c["shape"]
    Qs = c["Qs"]
    if rows_idx is not None:
        Qs = np.ascontiguousarray(Qs[:, rows_idx, :])
        O, m, l = O[:, rows_idx], m[:, rows_idx], l[:, rows_idx]
        sh = orc.shape(sh.hd, sh.nkv, len(rows_idx), sh.quant, sh.rs)
    O3, m3, l3 = orc.partial_f32(sh, Qs, c["K"], c["V"], nk)
    Of, mf, lf = orc.partial_f64(sh, Qs, c["K"], c["V"], nk)
    e32 = orc.rel_err(O, m, l, O3.astype(np.float64), m3.astype(np.float64), l3.astype(np.float64))
    e64 = orc.rel_err(O, m, l, Of, mf, lf)
    assert e32[0] <= TOL and e32[1] <= TOL, ("vs reference arithmetic", e32)
    assert e64[0] <= TOL_F64 and e64[1] <= TOL_F64, ("vs fp64", e64)
    # m is the row's exact maximum score (sme_attn_partial's m), not only a reference point for O and l
    assert np.abs(m - m3).max() <= TOL, ("m vs reference arithmetic", np.abs(m - m3).max())


def _case(ctx, c, shape, rows_idx=None):
    import torch
    nkv, rows, hd = shape.nkv, shape.rows, shape.hd
    n = c["K"].shape[0]
    K = torch.from_numpy(c["K"]).cuda()
    V = torch.from_numpy(c["V"]).cuda()
    Qs = torch.from_numpy(c["Qs"].view(np.int16)).cuda().view(torch.float16)
    O = torch.empty((nkv, rows, hd), device="cuda")
    m = torch.empty((nkv, rows), device="cuda")
    l = torch.empty_like(m)
    rc, why = _noalloc(shape, Qs, K, V, n, O, m, l)
    assert rc == 0, (rc, why)
    On, mn, ln = O.cpu().numpy(), m.cpu().numpy(), l.cpu().numpy()
    _vs_oracle(c, On, mn, ln, n, rows_idx)
    Oa, ma, la = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), n, 0)], 1)
    ctx.status()
    e = orc.rel_err(On, mn, ln, Oa[0].cpu().numpy().astype(np.float64), ma[0].cpu().numpy().astype(np.float64),
                    la[0].cpu().numpy().astype(np.float64))
    assert e[0] <= TOL and e[1] <= TOL, ("vs pa_cuda_attn", e)


@pytest.mark.parametrize("hd,nkv,rows,quant,nk", [(128, 8, 5, orc.Q8_0, 8192), (256, 4, 48, orc.Q4_0, 3000),
                                                  (128, 8, 5, orc.F16, 2000)])
def test_noalloc_matches_oracle_and_allocating_entry_two_calls(ctx, hd, nkv, rows, quant, nk):
    shape = pa.shape_for(hd, nkv, rows, quant)
    for call in range(2):
        c = orc.gen_case(500 + 17 * call + hd + quant, hd, nkv, rows, nk + 77 * call, quant)
        _case(ctx, c, shape)


def test_noalloc_partials_nearly_filling_the_fixed_array(ctx):
    # one chunk partial of 8 heads x 1,000 rows x 130 floats is 4.16 MB: 3 fit the 16 MiB array, so 65,536 keys run
    # as 3 chunks of ~22k keys (above the usual 16,384-key chunk cap); two calls in a row, rows sampled for the oracle
    hd, nkv, rows = 128, 8, 1000
    shape = pa.shape_for(hd, nkv, rows, pa.Q8_0)
    idx = np.array([0, 1, 7, 8, 333, 500, 998, 999])
    for call in range(2):
        c = orc.gen_case(900 + call, hd, nkv, rows, 65536 - 640 * call, orc.Q8_0)
        _case(ctx, c, shape, idx)


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch():
    import torch
    # one chunk partial of 8 heads x 4096 rows x 130 floats is 17 MB, beyond the 16 MiB array
    shape = pa.shape_for(128, 8, 4096, pa.Q8_0)
    t = torch.zeros(16, device="cuda")
    rc, why = _noalloc(shape, t, t, t, 64, t, t, t)
    assert rc == api.EUNSUPPORTED and "16 MiB" in why, (rc, why)
