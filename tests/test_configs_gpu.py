"""Each BASELINE configuration at its own size, on the GPU, against the oracle on identical seeded inputs.

Inputs follow the BASELINE distributions (Q ~ N(0,1); K, V ~ N(0,1) with 4 K channels per head x8; config 4's V
Student-t(3); Q8_0 or Q4_0 as the config says), generated on the device by the torch quantisers that
tests/test_oracle.py pins bit-for-bit to the oracle's. Where the full oracle would take minutes on the host, the GPU
still computes every row and the oracle checks a seeded sample of rows: rows are independent of one another in this
computation, so a sample is an exact check of those rows. Gate: 2e-3 on the merged, normalised output and on lse
against the oracle's restatement of the reference's arithmetic."""
import numpy as np
import pytest

import backburner_b200 as pa
from backburner_b200 import shard
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

TOL = 2e-3
NKV, GQA, HD = 8, 5, 128


def _kv(torch, seed, nk, quant, student_t=False):
    """K and V rows [nk][NKV*hb] with the BASELINE distributions, quantised on the device."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    kf = torch.randn((nk, NKV, HD), generator=g, device="cuda")
    for h in range(NKV):
        ch = torch.randperm(HD, generator=g, device="cuda")[:4]
        kf[:, h, ch] *= 8.0
    if student_t:
        z = torch.randn((nk, NKV, HD), generator=g, device="cuda")
        chi2 = sum(torch.randn((nk, NKV, HD), generator=g, device="cuda") ** 2 for _ in range(3))
        vf = z / torch.sqrt(chi2 / 3.0)
    else:
        vf = torch.randn((nk, NKV, HD), generator=g, device="cuda")
    qz = pa.quantize_q8_0 if quant == pa.Q8_0 else pa.quantize_q4_0
    return qz(kf).reshape(nk, -1).contiguous(), qz(vf).reshape(nk, -1).contiguous()


def _qs(torch, seed, rows):
    """f16(q * 1/sqrt(128)) [NKV][rows][HD] on the device, and the same bits on the host."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((NKV, rows, HD), generator=g, device="cuda")
    qs = (q * (1.0 / HD ** 0.5)).to(torch.float16)
    return qs, qs.cpu().view(torch.int16).numpy().view(np.uint16)


def _oracle_rows(Qs_host, sample, K_host, V_host, nk, quant):
    """The oracle's (O, m, l) for the sampled rows of every head (multi-threaded fp32 restatement)."""
    sub = np.ascontiguousarray(Qs_host[:, sample, :])
    sh = orc.shape(HD, NKV, len(sample), quant)
    return orc.partial_f32_mt(sh, sub, K_host, V_host, nk)


def _check(O, m, l, ref, sample):
    Or, mr, lr = ref
    e = orc.rel_err(O[:, sample], m[:, sample], l[:, sample], Or.astype(np.float64), mr.astype(np.float64),
                    lr.astype(np.float64))
    assert e[0] <= TOL and e[1] <= TOL, e
    valid = lr > 0
    dm = np.abs(m[:, sample].astype(np.float64) - mr.astype(np.float64))[valid].max() if valid.any() else 0.0
    assert dm <= TOL, ("m is not the row maximum", dm)
    return e


def test_config0_decode_folded_with_a_local_partial(ctx):
    """Config 0: 1 token (5 rows per KV head), 8,192 offloaded Q8_0 positions; the offloaded partial is folded by LSE
    into a second seeded partial over 1,024 local positions (the host's own, computed here by the oracle), as the
    host does with the engine's reply. Checked against the oracle over all 9,216 positions."""
    import torch
    rows = GQA
    K, V = _kv(torch, 11, 8192, pa.Q8_0)
    Kl, Vl = _kv(torch, 12, 1024, pa.Q8_0)
    Qs, Qs_h = _qs(torch, 13, rows)
    shape = pa.shape_for(HD, NKV, rows, pa.Q8_0)
    O, m, l = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), 8192, 0)])
    ctx.status()
    sh = orc.shape(HD, NKV, rows, orc.Q8_0)
    Kl_h, Vl_h = Kl.cpu().numpy(), Vl.cpu().numpy()
    Ol, ml, ll = orc.partial_f32(sh, Qs_h, Kl_h, Vl_h, 1024)
    out = (torch.from_numpy(Ol).cuda().reshape(-1, HD).contiguous(), torch.from_numpy(ml).cuda().reshape(-1).contiguous(),
           torch.from_numpy(ll).cuda().reshape(-1).contiguous())
    Om, mm, lm = pa.merge(ctx, HD, O.reshape(1, -1, HD), m.reshape(1, -1), l.reshape(1, -1), out=out, fold=True)
    ctx.status()
    Kall = np.concatenate([K.cpu().numpy(), Kl_h])
    Vall = np.concatenate([V.cpu().numpy(), Vl_h])
    Of, mf, lf = orc.partial_f64(sh, Qs_h, Kall, Vall, 9216)
    O3, m3, l3 = orc.partial_f32(sh, Qs_h, Kall, Vall, 9216)
    got = (Om.cpu().numpy().reshape(NKV, rows, HD), mm.cpu().numpy().reshape(NKV, rows), lm.cpu().numpy().reshape(NKV, rows))
    e32 = orc.rel_err(*got, O3.astype(np.float64), m3.astype(np.float64), l3.astype(np.float64))
    e64 = orc.rel_err(*got, Of, mf, lf)
    assert e32[0] <= TOL and e32[1] <= TOL, e32
    assert e64[0] <= 5e-3 and e64[1] <= 5e-3, e64   # pa-tool's own gate against exact arithmetic


def test_config2_prefill_full_layer(ctx):
    """Config 2: 512 tokens (2,560 rows per KV head) against 65,536 Q8_0 positions, one full layer on the tcgen05
    kernel; 48 sampled rows per head checked."""
    import torch
    rows, nk = 512 * GQA, 65536
    K, V = _kv(torch, 21, nk, pa.Q8_0)
    Qs, Qs_h = _qs(torch, 22, rows)
    shape = pa.shape_for(HD, NKV, rows, pa.Q8_0)
    O, m, l = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), nk, 0)])
    ctx.status()
    sample = np.sort(np.random.default_rng(23).choice(rows, 48, replace=False))
    ref = _oracle_rows(Qs_h, sample, K.cpu().numpy(), V.cpu().numpy(), nk, orc.Q8_0)
    _check(O[0].cpu().numpy(), m[0].cpu().numpy(), l[0].cpu().numpy(), ref, sample)


def test_config3_verify_batch_q4(ctx):
    """Config 3: 16 draft tokens (80 rows per KV head) against 196,608 Q4_0 positions, all visible (the causal mask
    among the new tokens belongs to the host's local partial); every row checked."""
    import torch
    rows, nk = 16 * GQA, 196608
    K, V = _kv(torch, 31, nk, pa.Q4_0)
    Qs, Qs_h = _qs(torch, 32, rows)
    shape = pa.shape_for(HD, NKV, rows, pa.Q4_0)
    O, m, l = pa.attn(ctx, shape, Qs, [pa.Seg(K.data_ptr(), V.data_ptr(), nk, 0)])
    ctx.status()
    sample = np.arange(rows)
    ref = _oracle_rows(Qs_h, sample, K.cpu().numpy(), V.cpu().numpy(), nk, orc.Q4_0)
    _check(O[0].cpu().numpy(), m[0].cpu().numpy(), l[0].cpu().numpy(), ref, sample)


@pytest.mark.parametrize("tokens", [1, 512])
def test_config4_uneven_shards_student_t(ctx, tokens):
    """Config 4: 229,376 Q8_0 positions with Student-t(3) V, split by position into 8 seeded uneven shards of 10-20%
    each; each shard's partial is packed as a rank's all-gather contribution and the packed set merged by
    pa_cuda_merge_gathered, for a 1-token decode and a 512-token prefill. Checked against the oracle over all
    positions (every row for decode, 32 sampled rows per head for prefill)."""
    import torch
    nk, world = 229376, 8
    rng = np.random.default_rng(41)
    w = rng.uniform(0.10, 0.20, world)
    shares = np.floor(w / w.sum() * nk).astype(int)
    shares[-1] += nk - shares.sum()
    assert shares.sum() == nk and shares.min() > 0
    rows = tokens * GQA
    K, V = _kv(torch, 42, nk, pa.Q8_0, student_t=True)
    Qs, Qs_h = _qs(torch, 43, rows)
    shape = pa.shape_for(HD, NKV, rows, pa.Q8_0)
    R = NKV * rows
    gathered = torch.empty((world, R * (HD + 2)), dtype=torch.float32, device="cuda")
    for r in range(world):
        k0, cnt = shard.shard_range(nk, world, r, [int(x) for x in shares])
        Op, mp, lp = pa.packed_views(gathered[r], R, HD)
        seg = pa.Seg(K.data_ptr() + k0 * shape.rs, V.data_ptr() + k0 * shape.rs, cnt, 0)
        pa.attn(ctx, shape, Qs, [seg], out=(Op.view(1, NKV, rows, HD), mp.view(1, NKV, rows), lp.view(1, NKV, rows)))
    O, m, l = pa.merge_gathered(ctx, HD, R, gathered, world)
    ctx.status()
    sample = np.arange(rows) if tokens == 1 else np.sort(rng.choice(rows, 32, replace=False))
    ref = _oracle_rows(Qs_h, sample, K.cpu().numpy(), V.cpu().numpy(), nk, orc.Q8_0)
    _check(O.cpu().numpy().reshape(NKV, rows, HD), m.cpu().numpy().reshape(NKV, rows), l.cpu().numpy().reshape(NKV, rows),
           ref, sample)
