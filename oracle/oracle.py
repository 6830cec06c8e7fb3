"""numpy/ctypes face of the oracle (liboracle.so, pa_oracle.c) and of the reference shim (_ref/libparef.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg, as the
checker. The product path (backburner_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libparef.so")
F16, Q8_0, Q4_0 = 0, 1, 2

_u8p = ctypes.POINTER(ctypes.c_uint8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


class _Shape(ctypes.Structure):
    _fields_ = [("hd", ctypes.c_int), ("nkv", ctypes.c_int), ("rows", ctypes.c_int), ("quant", ctypes.c_int),
                ("rs", ctypes.c_size_t), ("hb", ctypes.c_size_t)]


def build():
    """Compile liboracle.so if it is missing or older than its source."""
    src = os.path.join(HERE, "pa_oracle.c")
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB)
        L.orc_f2h.restype = ctypes.c_uint16
        L.orc_f2h.argtypes = [ctypes.c_float]
        L.orc_h2f.restype = ctypes.c_float
        L.orc_h2f.argtypes = [ctypes.c_uint16]
        L.orc_f2h_n.argtypes = [_f32p, _u16p, ctypes.c_size_t]
        L.orc_h2f_n.argtypes = [_u16p, _f32p, ctypes.c_size_t]
        L.orc_lcg_frand.restype = ctypes.c_float
        L.orc_lcg_frand.argtypes = [ctypes.POINTER(ctypes.c_uint64)]
        L.orc_pt_make_q8_row.argtypes = [_u8p, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_uint64)]
        L.orc_pt_make_q4_row.argtypes = [_u8p, ctypes.c_int, ctypes.c_float, ctypes.POINTER(ctypes.c_uint64)]
        L.orc_deq.restype = ctypes.c_float
        L.orc_deq.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_quant_q8_0.argtypes = [_f32p, ctypes.c_size_t, _u8p]
        L.orc_quant_q4_0.argtypes = [_f32p, ctypes.c_size_t, _u8p]
        L.orc_scale_q.argtypes = [_f32p, ctypes.c_float, _u16p, ctypes.c_size_t]
        L.orc_partial_f64.argtypes = [ctypes.POINTER(_Shape), _u16p, _u8p, _u8p, ctypes.c_uint32, _f64p, _f64p, _f64p]
        L.orc_partial_f32.argtypes = [ctypes.POINTER(_Shape), _u16p, _u8p, _u8p, ctypes.c_uint32, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p]
        L.orc_partial_f32_i8q.restype = ctypes.c_int
        L.orc_partial_f32_i8q.argtypes = [ctypes.POINTER(_Shape), _u16p, _u8p, _u8p, ctypes.c_uint32, ctypes.c_int,
                                          ctypes.c_int, ctypes.c_int, _f32p, _f32p, _f32p]
        L.orc_partial_f32_mt.restype = ctypes.c_int
        L.orc_partial_f32_mt.argtypes = [ctypes.POINTER(_Shape), _u16p, _u8p, _u8p, ctypes.c_uint32, ctypes.c_int,
                                         ctypes.c_uint32, _f32p, _f32p, _f32p]
        L.orc_merge_partial.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_size_t, ctypes.c_int]
        L.orc_merge_slots.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_size_t, ctypes.c_int, _f32p, _f32p,
                                      _f32p]
        L.orc_normalize.argtypes = [_f32p, _f32p, _f32p, ctypes.c_size_t, ctypes.c_int, _u16p, _f32p]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def head_bytes(quant, hd):
    return hd // 32 * (34 if quant == Q8_0 else 18) if quant in (Q8_0, Q4_0) else 2 * hd


def shape(hd, nkv, rows, quant=Q8_0, rs=None):
    hb = head_bytes(quant, hd)
    return _Shape(hd, nkv, rows, quant, rs if rs is not None else nkv * hb, hb)


# ------------------------------------------------------------------ formats
def f2h(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f2h_n(_p(x, _f32p), _p(out, _u16p), x.size)
    return out


def h2f(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_h2f_n(_p(h, _u16p), _p(out, _f32p), h.size)
    return out


def quant_q8_0(x: np.ndarray) -> np.ndarray:
    """[..., hd] float32 -> [..., hd/32*34] uint8"""
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, hd = x.shape
    out = np.empty((*lead, hd // 32 * 34), dtype=np.uint8)
    lib().orc_quant_q8_0(_p(x, _f32p), x.size // 32, _p(out, _u8p))
    return out


def quant_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    *lead, hd = x.shape
    out = np.empty((*lead, hd // 32 * 18), dtype=np.uint8)
    lib().orc_quant_q4_0(_p(x, _f32p), x.size // 32, _p(out, _u8p))
    return out


def quantize(x, quant):
    """[..., hd] float32 -> stored rows: Q8_0 / Q4_0 blocks, or f16 values (the storage of f16 pages)."""
    if quant == F16:
        h = f2h(x)
        return h.view(np.uint8).reshape(*h.shape[:-1], h.shape[-1] * 2)
    return quant_q8_0(x) if quant == Q8_0 else quant_q4_0(x)


def deq(row: np.ndarray, quant, hd, h, d) -> float:
    row = np.ascontiguousarray(row, dtype=np.uint8)
    return float(lib().orc_deq(_p(row, _u8p), quant, hd, h, d))


def scale_q(Q: np.ndarray, scale: float) -> np.ndarray:
    Q = np.ascontiguousarray(Q, dtype=np.float32)
    out = np.empty(Q.shape, dtype=np.uint16)
    lib().orc_scale_q(_p(Q, _f32p), scale, _p(out, _u16p), Q.size)
    return out


def lcg_seq(seed: int, n: int) -> np.ndarray:
    s = ctypes.c_uint64(seed)
    return np.array([lib().orc_lcg_frand(ctypes.byref(s)) for _ in range(n)], dtype=np.float32)


def pt_make_rows(seed: int, q4: bool, n: int, nkv: int, amp: float) -> np.ndarray:
    """pa-tool's test rows (HD 256): n rows of nkv heads from LCG state `seed`."""
    rs = nkv * (144 if q4 else 272)
    out = np.zeros((n, rs), dtype=np.uint8)
    s = ctypes.c_uint64(seed)
    fn = lib().orc_pt_make_q4_row if q4 else lib().orc_pt_make_q8_row
    for j in range(n):
        fn(out[j].ctypes.data_as(_u8p), nkv, amp, ctypes.byref(s))
    return out


# ------------------------------------------------------------------ partials
def partial_f64(sh: _Shape, Qs: np.ndarray, K: np.ndarray, V: np.ndarray, nk: int):
    """fp64 reference partial: returns (O [nkv][rows][hd], m [nkv][rows], l [nkv][rows]) float64."""
    Qs = np.ascontiguousarray(Qs, dtype=np.uint16)
    K = np.ascontiguousarray(K, dtype=np.uint8)
    V = np.ascontiguousarray(V, dtype=np.uint8)
    O = np.empty((sh.nkv, sh.rows, sh.hd), dtype=np.float64)
    m = np.empty((sh.nkv, sh.rows), dtype=np.float64)
    l = np.empty_like(m)
    lib().orc_partial_f64(ctypes.byref(sh), _p(Qs, _u16p), _p(K, _u8p), _p(V, _u8p), nk, _p(O, _f64p), _p(m, _f64p),
                          _p(l, _f64p))
    return O, m, l


def partial_f32(sh: _Shape, Qs, K, V, nk: int, bk: int = 512):
    Qs = np.ascontiguousarray(Qs, dtype=np.uint16)
    K = np.ascontiguousarray(K, dtype=np.uint8)
    V = np.ascontiguousarray(V, dtype=np.uint8)
    O = np.empty((sh.nkv, sh.rows, sh.hd), dtype=np.float32)
    m = np.empty((sh.nkv, sh.rows), dtype=np.float32)
    l = np.empty_like(m)
    lib().orc_partial_f32(ctypes.byref(sh), _p(Qs, _u16p), _p(K, _u8p), _p(V, _u8p), nk, bk, 0, sh.nkv, _p(O, _f32p),
                          _p(m, _f32p), _p(l, _f32p))
    return O, m, l


def partial_f32_i8q(sh: _Shape, Qs, K, V, nk: int, bk: int = 512):
    """orc_partial_f32 with the reference's int8-domain QK (scripts/sme/sme_attn.c:465-508); Q8_0 rows only."""
    Qs = np.ascontiguousarray(Qs, dtype=np.uint16)
    K = np.ascontiguousarray(K, dtype=np.uint8)
    V = np.ascontiguousarray(V, dtype=np.uint8)
    O = np.empty((sh.nkv, sh.rows, sh.hd), dtype=np.float32)
    m = np.empty((sh.nkv, sh.rows), dtype=np.float32)
    l = np.empty_like(m)
    rc = lib().orc_partial_f32_i8q(ctypes.byref(sh), _p(Qs, _u16p), _p(K, _u8p), _p(V, _u8p), nk, bk, 0, sh.nkv,
                                   _p(O, _f32p), _p(m, _f32p), _p(l, _f32p))
    if rc != 0:
        raise ValueError("the int8-domain QK needs Q8_0 rows")
    return O, m, l


def partial_f32_mt(sh: _Shape, Qs, K, V, nk: int, nthreads: int = 0, chunk_keys: int = 4096):
    Qs = np.ascontiguousarray(Qs, dtype=np.uint16)
    K = np.ascontiguousarray(K, dtype=np.uint8)
    V = np.ascontiguousarray(V, dtype=np.uint8)
    O = np.empty((sh.nkv, sh.rows, sh.hd), dtype=np.float32)
    m = np.empty((sh.nkv, sh.rows), dtype=np.float32)
    l = np.empty_like(m)
    rc = lib().orc_partial_f32_mt(ctypes.byref(sh), _p(Qs, _u16p), _p(K, _u8p), _p(V, _u8p), nk,
                                  nthreads or os.cpu_count() or 1, chunk_keys, _p(O, _f32p), _p(m, _f32p), _p(l, _f32p))
    if rc != 0:
        raise MemoryError("orc_partial_f32_mt")
    return O, m, l


def merge_partial(O, m, l, O2, m2, l2):
    """in-place merge_partial (phone-attn.h:231-239) on float32 arrays [rows][hd], [rows]"""
    rows, hd = m.size, O.shape[-1]
    lib().orc_merge_partial(_p(O, _f32p), _p(m, _f32p), _p(l, _f32p), _p(np.ascontiguousarray(O2, np.float32), _f32p),
                            _p(np.ascontiguousarray(m2, np.float32), _f32p),
                            _p(np.ascontiguousarray(l2, np.float32), _f32p), rows, hd)


def merge_slots(Op, mp, lp):
    """[n][rows][hd], [n][rows] -> (O, m, l) (pa_merge semantics)"""
    Op = np.ascontiguousarray(Op, np.float32)
    mp = np.ascontiguousarray(mp, np.float32)
    lp = np.ascontiguousarray(lp, np.float32)
    n, rows, hd = Op.shape
    O = np.empty((rows, hd), np.float32)
    m = np.empty((rows,), np.float32)
    l = np.empty_like(m)
    lib().orc_merge_slots(_p(Op, _f32p), _p(mp, _f32p), _p(lp, _f32p), n, rows, hd, _p(O, _f32p), _p(m, _f32p),
                          _p(l, _f32p))
    return O, m, l


def normalize(O, m, l):
    O = np.ascontiguousarray(O, np.float32)
    m = np.ascontiguousarray(m, np.float32)
    l = np.ascontiguousarray(l, np.float32)
    hd = O.shape[-1]
    rows = m.size
    Oh = np.empty((rows, hd), np.uint16)
    lse = np.empty((rows,), np.float32)
    lib().orc_normalize(_p(O, _f32p), _p(m, _f32p), _p(l, _f32p), rows, hd, _p(Oh, _u16p), _p(lse, _f32p))
    return Oh, lse


def reexpand(Oh, lse):
    """A normalised reply row as the host's co-attention slot (phone-attn.h:18-20: "O_unnorm = O, S = 1, M = lse"):
    (O = f32(Oh), m = lse, l = 1), or l = 0 for a reply with no keys (lse = -inf)."""
    lse = np.ascontiguousarray(lse, np.float32)
    O = h2f(np.ascontiguousarray(Oh, np.uint16)).astype(np.float32)
    l = np.where(lse > -np.inf, 1.0, 0.0).astype(np.float32)
    return O, lse.copy(), l


def fold_reply(O, m, l, Oh, lse):
    """The host's fold of a normalised reply into its unnormalised partial (O, m, l), in place: merge_partial
    (phone-attn.h:231-239) of the re-expanded reply."""
    O2, m2, l2 = reexpand(Oh, lse)
    merge_partial(O, m, l, O2.reshape(O.shape), m2.reshape(m.shape), l2.reshape(l.shape))


# ------------------------------------------------------------------ synthetic inputs
def gen_case(seed: int, hd: int, nkv: int, rows: int, nk: int, quant=Q8_0, outliers: int = 4, student_t: bool = False,
             scale: float | None = None):
    """Seeded synthetic case with the BASELINE distributions: Q ~ N(0,1); K, V ~ N(0,1) with `outliers` K channels
    per head x8; V optionally Student-t(3). Returns dict(Q fp32 [nkv][rows][hd], Qs f16 bits, K, V uint8 rows, scale)."""
    rng = np.random.default_rng(seed)
    Q = rng.standard_normal((nkv, rows, hd), dtype=np.float32)
    Kf = rng.standard_normal((nk, nkv, hd), dtype=np.float32)
    for h in range(nkv):
        ch = rng.choice(hd, size=outliers, replace=False) if outliers else []
        Kf[:, h, ch] *= 8.0
    Vf = (rng.standard_t(3, size=(nk, nkv, hd)).astype(np.float32) if student_t
          else rng.standard_normal((nk, nkv, hd), dtype=np.float32))
    K = quantize(Kf, quant).reshape(nk, nkv * head_bytes(quant, hd))
    V = quantize(Vf, quant).reshape(nk, nkv * head_bytes(quant, hd))
    sc = 1.0 / np.sqrt(hd) if scale is None else scale
    return dict(Q=Q, Qs=scale_q(Q, sc), K=K, V=V, scale=sc, shape=shape(hd, nkv, rows, quant))


def rel_err(O, m, l, Oref, mref, lref):
    """max |O/l - Oref/lref| / max |Oref/lref| over rows with keys, and max |lse - lse_ref|."""
    O = np.asarray(O, np.float64)
    l = np.asarray(l, np.float64)
    m = np.asarray(m, np.float64)
    on = O / np.where(l > 0, l, 1)[..., None]
    rn = Oref / np.where(lref > 0, lref, 1)[..., None]
    valid = lref > 0
    if not valid.any():
        return 0.0, 0.0
    eo = np.abs(on - rn)[valid].max() / max(np.abs(rn[valid]).max(), 1e-30)
    lse = m + np.log(np.where(l > 0, l, 1))
    lse_ref = mref + np.log(np.where(lref > 0, lref, 1))
    el = np.abs(lse - lse_ref)[valid].max()
    return float(eo), float(el)


# ------------------------------------------------------------------ the reference shim (_ref/libparef.so)
_ref = None


def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref():
    """The reference's own helpers compiled from its sources (see ref_shim.cpp); raises if not built."""
    global _ref
    if _ref is None:
        L = ctypes.CDLL(REF_LIB)
        L.ref_frand_seq.argtypes = [ctypes.c_uint64, _f32p, ctypes.c_int]
        L.ref_make_rows.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _u8p]
        L.ref_deq.restype = ctypes.c_float
        L.ref_deq.argtypes = [_u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.ref_f2h.restype = ctypes.c_uint16
        L.ref_f2h.argtypes = [ctypes.c_float]
        L.ref_h2f.restype = ctypes.c_float
        L.ref_h2f.argtypes = [ctypes.c_uint16]
        L.ref_merge_partial.argtypes = [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, ctypes.c_size_t]
        _ref = L
    return _ref
