"""The oracle restatement pinned against the reference's own code: golden vectors written by the reference's
pa-tool helpers and merge_partial (tests/golden/make_golden.py), and, where the reference tree was built into
oracle/_ref, the reference's own `pa-tool test` fp64 gate run against the oracle behind the reference's server."""
import os
import socket
import subprocess
import time

import numpy as np
import pytest

from oracle import oracle as orc

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_vectors.npz"))


def test_f2h_matches_reference_and_ieee():
    xs = GOLD["f2h_in"]
    assert np.array_equal(orc.f2h(xs), GOLD["f2h_out"])
    with np.errstate(over="ignore"):
        assert np.array_equal(orc.f2h(xs), xs.astype(np.float16).view(np.uint16))
    rng = np.random.default_rng(1)
    ys = (rng.standard_normal(200000) * 10.0 ** rng.integers(-8, 5, 200000)).astype(np.float32)
    assert np.array_equal(orc.f2h(ys), ys.astype(np.float16).view(np.uint16))


def test_h2f_all_halves():
    hs = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = orc.h2f(hs).view(np.uint32)
    ref = GOLD["h2f_out"].view(np.uint32)
    nan = np.isnan(GOLD["h2f_out"])
    assert np.array_equal(got[~nan], ref[~nan])
    assert np.isnan(orc.h2f(hs)[nan]).all()
    assert np.array_equal(orc.h2f(hs)[~nan], hs.view(np.float16).astype(np.float32)[~nan])


def test_lcg_matches_pa_tool():
    seq = orc.lcg_seq(int(GOLD["lcg_seed"][0]), len(GOLD["lcg_seq"]))
    assert np.array_equal(seq, GOLD["lcg_seq"])


@pytest.mark.parametrize("q4", [False, True])
def test_pa_tool_rows_and_deq(q4):
    tag = "q4" if q4 else "q8"
    rows = orc.pt_make_rows(12345, q4, 6, 4, 1.5)
    assert np.array_equal(rows, GOLD[f"rows_{tag}"])
    quant = orc.Q4_0 if q4 else orc.Q8_0
    deq = np.array([[orc.deq(rows[j], quant, 256, h, d) for h in range(4) for d in range(256)] for j in range(6)],
                   np.float32)
    assert np.array_equal(deq, GOLD[f"deq_{tag}"])


def test_merge_partial_matches_reference():
    rows, hd = 6, 256
    x = GOLD["merge_in"]
    o = 0
    O = x[o:o + rows * hd].reshape(rows, hd).copy(); o += rows * hd
    m = x[o:o + rows].copy(); o += rows
    l = x[o:o + rows].copy(); o += rows
    O2 = x[o:o + rows * hd].reshape(rows, hd).copy(); o += rows * hd
    m2 = x[o:o + rows].copy(); o += rows
    l2 = x[o:o + rows].copy()
    orc.merge_partial(O, m, l, O2, m2, l2)
    ref = GOLD["merge_out"]
    np.testing.assert_allclose(O.ravel(), ref[:rows * hd], rtol=2e-6, atol=1e-6)
    np.testing.assert_allclose(m, ref[rows * hd:rows * hd + rows], rtol=0, atol=0)
    np.testing.assert_allclose(l, ref[rows * hd + rows:], rtol=2e-6)


@pytest.mark.skipif(not orc.ref_available(), reason="oracle/_ref not built (needs the reference tree)")
def test_live_reference_shim_agrees():
    import ctypes
    R = orc.ref()
    rng = np.random.default_rng(3)
    xs = rng.standard_normal(5000).astype(np.float32) * 300
    assert np.array_equal(orc.f2h(xs), np.array([R.ref_f2h(float(v)) for v in xs], np.uint16))
    rows = np.zeros((3, 4 * 272), np.uint8)
    R.ref_make_rows(99, 0, 3, 4, 2.0, rows.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    assert np.array_equal(rows, orc.pt_make_rows(99, False, 3, 4, 2.0))


@pytest.mark.parametrize("hd,nkv,rows,quant,nk", [
    (128, 8, 5, orc.Q8_0, 1000), (128, 8, 5, orc.Q4_0, 777), (256, 4, 48, orc.Q8_0, 300),
    (256, 4, 12, orc.Q4_0, 513), (128, 2, 80, orc.Q8_0, 64), (128, 8, 5, orc.Q8_0, 1), (128, 8, 5, orc.F16, 600),
    (256, 4, 48, orc.F16, 129)])
def test_f32_block_online_matches_f64(hd, nkv, rows, quant, nk):
    c = orc.gen_case(hd * 7 + nk, hd, nkv, rows, nk, quant)
    sh = c["shape"]
    Of, mf, lf = orc.partial_f64(sh, c["Qs"], c["K"], c["V"], nk)
    O3, m3, l3 = orc.partial_f32(sh, c["Qs"], c["K"], c["V"], nk)
    eo, el = orc.rel_err(O3, m3, l3, Of, mf, lf)
    assert eo < 5e-3 and el < 5e-3, (eo, el)
    np.testing.assert_allclose(m3, mf, atol=5e-3)   # K rounded to f16 moves scores by ~|s| * 2^-11


def test_f32_mt_matches_single_thread():
    c = orc.gen_case(5, 128, 8, 5, 5000, orc.Q8_0)
    sh = c["shape"]
    O1, m1, l1 = orc.partial_f32(sh, c["Qs"], c["K"], c["V"], 5000)
    for chunk in (512, 1024, 4096, 8192):
        O2, m2, l2 = orc.partial_f32_mt(sh, c["Qs"], c["K"], c["V"], 5000, nthreads=4, chunk_keys=chunk)
        eo, el = orc.rel_err(O2, m2, l2, O1.astype(np.float64), m1.astype(np.float64), l1.astype(np.float64))
        # P is rounded to f16 against each chunk's running max, so chunkings differ by ~2^-11 in O
        assert eo < 5e-4 and el < 1e-5, (chunk, eo, el)


def test_empty_partial_and_merge_conventions():
    c = orc.gen_case(1, 128, 2, 5, 0, orc.Q8_0)
    O, m, l = orc.partial_f64(c["shape"], c["Qs"], c["K"], c["V"], 0)
    assert np.all(l == 0) and np.all(np.isneginf(m)) and np.all(O == 0)
    Oh, lse = orc.normalize(np.zeros((2, 128), np.float32), np.full(2, -np.inf, np.float32), np.zeros(2, np.float32))
    assert np.all(Oh == 0) and np.all(np.isneginf(lse))


def test_reply_fold_equals_merging_the_partials():
    """The host's co-attention fold of a normalised reply (phone-attn.h:18-20: O_unnorm = O, S = 1, M = lse) gives the
    merge of the unnormalised partials (phone-attn.h:231-239), up to the reply's f16 rounding of O/l; a reply with no
    keys (lse = -inf) leaves the host's partial as it is, and a host row with no keys takes the reply."""
    c = orc.gen_case(808, 128, 2, 10, 3000, orc.Q8_0)
    sh = c["shape"]
    na = 1900
    OA, mA, lA = orc.partial_f32(sh, c["Qs"], c["K"][:na], c["V"][:na], na)
    OB, mB, lB = orc.partial_f32(sh, c["Qs"], c["K"][na:], c["V"][na:], 3000 - na)
    O1, m1, l1 = OB.copy(), mB.copy(), lB.copy()
    orc.merge_partial(O1, m1, l1, OA, mA, lA)
    Oh, lse = orc.normalize(OA, mA, lA)
    lse = lse.reshape(mA.shape)
    lse[0, 3] = -np.inf                     # the reply has no keys for this row
    O2, m2, l2 = OB.copy(), mB.copy(), lB.copy()
    l2[1, 4] = 0.0                          # the host has none for this one
    orc.fold_reply(O2, m2, l2, Oh.reshape(OA.shape), lse)
    Oh1, lse1 = orc.normalize(O1, m1, l1)
    Oh2, lse2 = orc.normalize(O2, m2, l2)
    Oh1, Oh2 = orc.h2f(Oh1).reshape(OA.shape), orc.h2f(Oh2).reshape(OA.shape)
    lse1, lse2 = lse1.reshape(mA.shape), lse2.reshape(mA.shape)
    ok = np.ones(mA.shape, bool)
    ok[0, 3] = ok[1, 4] = False
    assert np.abs(Oh2 - Oh1)[ok].max() <= 1e-3 * np.abs(Oh1).max()
    assert np.abs(lse2 - lse1)[ok].max() <= 1e-5 * np.abs(lse1).max()
    OBh, lseB = orc.normalize(OB, mB, lB)
    assert np.array_equal(Oh2[0, 3], orc.h2f(OBh).reshape(OA.shape)[0, 3]) and lse2[0, 3] == lseB.reshape(mA.shape)[0, 3]
    assert np.allclose(Oh2[1, 4], orc.h2f(Oh).reshape(OA.shape)[1, 4], rtol=1e-3, atol=1e-4)
    assert abs(lse2[1, 4] - lse[1, 4]) <= 1e-6


def test_merge_slots_equals_whole():
    c = orc.gen_case(11, 128, 8, 5, 3000, orc.Q8_0)
    sh = c["shape"]
    Ow, mw, lw = orc.partial_f64(sh, c["Qs"], c["K"], c["V"], 3000)
    parts = []
    for a, b in [(0, 1000), (1000, 1000), (1000, 2999), (2999, 3000)]:   # includes an empty part
        O, m, l = orc.partial_f32(sh, c["Qs"], c["K"][a:], c["V"][a:], b - a)
        if b == a:
            m[:] = -np.inf
        parts.append((O.reshape(-1, 128), m.ravel(), l.ravel()))
    O, m, l = orc.merge_slots(np.stack([p[0] for p in parts]), np.stack([p[1] for p in parts]),
                              np.stack([p[2] for p in parts]))
    # against fp64 with exact dequant: the f16 rounding of K, V and P (the reference's semantics) costs ~2e-3;
    # the reference's own gate is 5e-3 (phone-attn/pa-tool.cpp:173)
    eo, el = orc.rel_err(O, m, l, Ow.reshape(-1, 128), mw.ravel(), lw.ravel())
    assert eo < 5e-3 and el < 5e-3
    O1, m1, l1 = orc.partial_f32(sh, c["Qs"], c["K"], c["V"], 3000)
    eo, el = orc.rel_err(O, m, l, O1.reshape(-1, 128).astype(np.float64), m1.ravel().astype(np.float64),
                         l1.ravel().astype(np.float64))
    assert eo < 5e-4 and el < 1e-5


@pytest.mark.parametrize("quant", [orc.Q8_0, orc.Q4_0])
def test_torch_quantizers_match_oracle(quant):
    import torch
    from backburner_b200 import formats
    rng = np.random.default_rng(quant)
    x = rng.standard_normal((37, 8, 128)).astype(np.float32) * 3
    x[0, 0, :32] = 0.0                       # an all-zero block
    x[1, 2, 5] = 1e4                          # a large outlier
    ref = orc.quantize(x, quant)
    got = (formats.quantize_q8_0 if quant == orc.Q8_0 else formats.quantize_q4_0)(torch.from_numpy(x)).numpy()
    assert np.array_equal(got, ref)
    deq = formats.dequantize(torch.from_numpy(ref), quant, 128).numpy()
    want = np.array([orc.deq(ref[3, 1], quant, 128, 0, d) for d in range(128)], np.float32)
    assert np.array_equal(deq[3, 1], want)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.skipif(not os.path.exists(os.path.join(orc.HERE, "_ref", "pa-serve-oracle")),
                    reason="oracle/_ref not built (needs the reference tree)")
@pytest.mark.parametrize("env,extra", [({}, []), ({"PA_Q4": "1"}, []), ({"PA_NTOK": "1"}, []), ({"PA_BIG_TOK": "16"}, []),
                                       ({}, ["1", "1", "0", "1024", "1"])])
def test_reference_pa_tool_gate_passes_on_oracle(env, extra):
    """The reference's own `pa-tool test` (its fp64 check, 5e-3 gate) against the reference's pa::server with the
    oracle's fp32 path as the engine; the last case has the server keep the rows as f16 pages (store_f16,
    phone-attn/phone-attn.h:298-319)."""
    port = _free_port()
    srv = subprocess.Popen([os.path.join(orc.HERE, "_ref", "pa-serve-oracle"), str(port), "2"],
                           stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    try:
        time.sleep(0.3)
        e = dict(os.environ, **env)
        out = subprocess.run([os.path.join(orc.HERE, "_ref", "pa-tool"), "test", "127.0.0.1", str(port), "2048", "2",
                              "2", *extra], env=e, capture_output=True, text=True, timeout=120)
        text = out.stdout + out.stderr
        assert out.returncode == 0, text
        assert "-> PASS" in text and "FAIL" not in text, text
    finally:
        srv.kill()
        srv.wait()


def test_int8_domain_qk_error_against_fp64():
    """The reference's int8-domain QK (scripts/sme/sme_attn.c:465-508: sme_qk_i8blk's per-block int32 dot products of
    int8 Q and q8_0 K, combined by i8_combine as sum_b float(T_b) dq_b dk_b), with Q quantised per 32-block by the Q8_0
    rule, measured against the fp64 oracle with the reference's check metrics (sme_attn.c:768-772: per-row O/l error,
    m error, l error). On the BASELINE distributions its O error is ~1e-2: past pa-tool's 5e-3 gate and the 2e-3
    north-star tolerance, where the f16-domain QK the kernels use stays within both; this is why the CUDA path keeps Q
    in f16 by default and offers the int8 variant only as an opt-in mode (a bench-only kernel in the reference)."""
    for hd, nkv, rows, nk, seed in [(128, 8, 5, 8192, 1), (256, 4, 48, 4096, 3)]:
        c = orc.gen_case(seed, hd, nkv, rows, nk, orc.Q8_0)
        Of, mf, lf = orc.partial_f64(c["shape"], c["Qs"], c["K"], c["V"], nk)
        O1, m1, l1 = orc.partial_f32(c["shape"], c["Qs"], c["K"], c["V"], nk)
        O2, m2, l2 = orc.partial_f32_i8q(c["shape"], c["Qs"], c["K"], c["V"], nk)
        e16, e8 = orc.rel_err(O1, m1, l1, Of, mf, lf), orc.rel_err(O2, m2, l2, Of, mf, lf)
        assert e16[0] <= 2e-3 and e16[1] <= 2e-3, e16
        assert e8[0] > 3e-3 and e8[1] > 5e-3, e8
        assert np.abs(m2 - mf).max() > 1e-2 > np.abs(m1 - mf).max()
