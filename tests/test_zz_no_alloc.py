"""The allocation-free entry point (pa_cuda_attn_noalloc), called through the C ABI.

Some callers cannot allocate device memory themselves: a host runtime that owns all device memory in its own pool, or
an inference server that has reserved the GPU up front, cannot create a context or a plan, because both allocate
scratch. pa_cuda_attn_noalloc runs the same split-K kernel and merge on a fixed device array compiled into the library.
Here two calls in a row (different inputs, so the second cannot pass on the first call's leftovers) must match the
allocating entry point, pa_cuda_attn, within the tolerance of the other parity tests. The file is named to be
collected last and needs nothing from the other test files, so it passes alone in a fresh process too."""
import ctypes

import numpy as np
import pytest

import backburner_b200 as pa
from backburner_b200 import api
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL = 2e-3   # the parity tolerance of the other GPU tests


def _noalloc(shape, Qs, K, V, nk, O, m, l):
    why = ctypes.c_char_p()
    sh = shape.c()
    rc = pa.lib().pa_cuda_attn_noalloc(ctypes.byref(sh), Qs.data_ptr(), K.data_ptr(), V.data_ptr(), nk, O.data_ptr(),
                                       m.data_ptr(), l.data_ptr(), api._stream_ptr(None), ctypes.byref(why))
    return rc, (why.value or b"").decode()


@pytest.mark.parametrize("hd,nkv,rows,quant,nk", [(128, 8, 5, orc.Q8_0, 8192), (256, 4, 48, orc.Q4_0, 3000)])
def test_noalloc_matches_allocating_entry_two_calls(ctx, hd, nkv, rows, quant, nk):
    import torch
    shape = pa.shape_for(hd, nkv, rows, quant)
    for call in range(2):
        c = orc.gen_case(500 + 17 * call + hd, hd, nkv, rows, nk + 77 * call, quant)
        n = c["K"].shape[0]
        K = torch.from_numpy(c["K"]).cuda()
        V = torch.from_numpy(c["V"]).cuda()
        Qs = torch.from_numpy(c["Qs"].view(np.int16)).cuda().view(torch.float16)
        O = torch.empty((nkv, rows, hd), device="cuda")
        m = torch.empty((nkv, rows), device="cuda")
        l = torch.empty_like(m)
        rc, why = _noalloc(shape, Qs, K, V, n, O, m, l)
        assert rc == 0, (rc, why)
        Oa, ma, la = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), n, 0)], 1)
        ctx.status()
        e = orc.rel_err(O.cpu().numpy(), m.cpu().numpy(), l.cpu().numpy(), Oa[0].cpu().numpy().astype(np.float64),
                        ma[0].cpu().numpy().astype(np.float64), la[0].cpu().numpy().astype(np.float64))
        assert e[0] <= TOL and e[1] <= TOL, (call, e)


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch():
    import torch
    # one chunk partial of 8 heads x 4096 rows x 130 floats is 17 MB, beyond the 16 MiB array
    shape = pa.shape_for(128, 8, 4096, pa.Q8_0)
    t = torch.zeros(16, device="cuda")
    rc, why = _noalloc(shape, t, t, t, 64, t, t, t)
    assert rc == api.EUNSUPPORTED and "16 MiB" in why, (rc, why)
