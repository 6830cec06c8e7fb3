"""ctypes binding of libpacuda.so (include/pa_cuda.h) and the Python host API over it.

Tensors passed in are torch CUDA tensors (device memory, streams); nothing here computes attention itself.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Sequence

F16, Q8_0, Q4_0 = 0, 1, 2          # config_req.is_q8 (phone-attn/phone-attn.h:15)
QK_F16, QK_INT8 = 0, 1             # QK arithmetic: f16(d*q) K, or the int8-domain QK (scripts/sme/sme_attn.c:465-508)
_HERE = os.path.dirname(os.path.abspath(__file__))
lib_path = os.path.join(_HERE, "libpacuda.so")

OK, EINVAL, ECUDA, ENOMEM, ETIMEOUT, EUNSUPPORTED, ENCCL = 0, -1, -2, -3, -4, -5, -6


class PaCudaError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"pa_cuda error {code}: {msg}")
        self.code = code


class LibraryMissing(PaCudaError):
    def __init__(self, why: str):
        super().__init__(ECUDA, f"libpacuda.so not loadable ({why}); build it with `python -m backburner_b200.build`")


class _Shape(ctypes.Structure):
    _fields_ = [("hd", ctypes.c_uint32), ("nkv", ctypes.c_uint32), ("rows", ctypes.c_uint32),
                ("quant", ctypes.c_uint32), ("rs", ctypes.c_uint64), ("hb", ctypes.c_uint64)]


class _Seg(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("nk", ctypes.c_uint32), ("set", ctypes.c_uint32)]


class _Page(ctypes.Structure):
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("hk", ctypes.c_void_p), ("hv", ctypes.c_void_p)]


_P = ctypes.c_void_p
_SIGS = {
    "pa_cuda_available": (ctypes.c_int, []),
    "pa_cuda_abi_version": (ctypes.c_int, []),
    "pa_cuda_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(_P)]),
    "pa_cuda_destroy": (None, [_P]),
    "pa_cuda_last_error": (ctypes.c_char_p, [_P]),
    "pa_cuda_status": (ctypes.c_int, [_P, _P]),
    "pa_cuda_set_timeout_ns": (None, [_P, ctypes.c_uint64]),
    "pa_cuda_launch_count": (ctypes.c_uint64, [_P]),
    "pa_cuda_set_stall_test": (None, [_P, ctypes.c_int]),
    "pa_cuda_set_kernel": (None, [_P, ctypes.c_int]),
    "pa_cuda_set_qk_domain": (None, [_P, ctypes.c_int]),
    "pa_cuda_plan_create": (ctypes.c_int, [_P, ctypes.POINTER(_Shape), ctypes.c_uint32, ctypes.POINTER(_Seg),
                                           ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(_P)]),
    "pa_cuda_plan_scratch_bytes": (ctypes.c_size_t, [_P]),
    "pa_cuda_plan_jobs": (ctypes.c_uint32, [_P]),
    "pa_cuda_plan_launches": (ctypes.c_uint32, [_P]),
    "pa_cuda_plan_kernel": (ctypes.c_char_p, [_P]),
    "pa_cuda_plan_run": (ctypes.c_int, [_P, _P, _P, _P, _P, _P]),
    "pa_cuda_plan_run_host": (ctypes.c_int, [_P, _P, _P, _P, _P, _P]),
    "pa_cuda_plan_destroy": (None, [_P]),
    "pa_cuda_plan_profile": (ctypes.c_int, [_P, ctypes.c_uint32]),
    "pa_cuda_plan_kernel_ms": (ctypes.c_int, [_P, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint32)]),
    "pa_cuda_attn": (ctypes.c_int, [_P, ctypes.POINTER(_Shape), _P, ctypes.c_uint32, ctypes.POINTER(_Seg),
                                    ctypes.c_uint32, _P, _P, _P, _P]),
    "pa_cuda_attn_partial": (ctypes.c_int, [_P, ctypes.POINTER(_Shape), _P, ctypes.c_float, _P, _P, ctypes.c_uint32,
                                            _P, _P, _P, _P]),
    "pa_cuda_merge": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, _P, _P, _P, _P, _P, _P,
                                     ctypes.c_int, _P]),
    "pa_cuda_merge_gathered": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32, _P, _P, _P, _P,
                                              ctypes.c_int, _P]),
    "pa_cuda_normalize": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint64, _P, _P, _P, _P, _P, _P]),
    "pa_cuda_scale_q": (ctypes.c_int, [_P, _P, ctypes.c_float, ctypes.c_uint64, _P, _P]),
    "pa_cuda_fold_reply": (ctypes.c_int, [_P, ctypes.c_uint32, ctypes.c_uint64, _P, _P, _P, _P, _P, _P]),
    "pa_cuda_nccl_unique_id": (ctypes.c_int, [_P, ctypes.c_size_t]),
    "pa_cuda_nccl_comm_create": (ctypes.c_int, [_P, _P, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p)]),
    "pa_cuda_nccl_comm_destroy": (None, [_P]),
    "pa_cuda_shard_attn_allgather_merge": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _P]),
    "pa_cuda_set_shard_exchange": (None, [_P, ctypes.c_int]),
    "pa_cuda_shard_last": (None, [_P, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int)]),
    "pa_cuda_set_shard_groups": (None, [_P, ctypes.c_int]),
    "pa_cuda_set_shard_timeout_ms": (None, [_P, ctypes.c_uint32]),
    "pa_cuda_nccl_wait": (ctypes.c_int, [_P, _P, _P, ctypes.c_uint32]),
    "pa_cuda_alloc_page": (ctypes.c_int, [_P, ctypes.c_size_t, ctypes.POINTER(_Page)]),
    "pa_cuda_free_page": (None, [_P, ctypes.POINTER(_Page)]),
    "pa_cuda_begin": (ctypes.c_int, [_P, ctypes.POINTER(_Page), ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, _P,
                                     ctypes.POINTER(_Shape), ctypes.c_int, ctypes.c_int]),
    "pa_cuda_end": (ctypes.c_double, [_P, _P, _P, _P]),
    "pa_cuda_exec_ms": (ctypes.c_double, [_P]),
    "pa_cuda_arm": (ctypes.c_int, [_P, _P, ctypes.POINTER(ctypes.c_uint32), ctypes.c_int, ctypes.POINTER(_Shape),
                                   ctypes.c_int]),
    "pa_cuda_graph_calls": (ctypes.c_uint64, [_P]),
    "pa_cuda_attn_noalloc": (ctypes.c_int, [ctypes.POINTER(_Shape), _P, _P, _P, ctypes.c_uint32, _P, _P, _P, _P,
                                            ctypes.POINTER(ctypes.c_char_p)]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded libpacuda.so (raises LibraryMissing if it is not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(lib_path):
            raise LibraryMissing("not built")
        try:
            L = ctypes.CDLL(lib_path)
        except OSError as e:  # pragma: no cover - depends on the machine
            raise LibraryMissing(str(e)) from e
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def available() -> bool:
    """True when libpacuda.so loads and a compute-capability-10 GPU is visible (pa_cuda_available)."""
    try:
        return bool(lib().pa_cuda_available())
    except LibraryMissing:
        return False


def head_bytes(quant: int, hd: int) -> int:
    return hd // 32 * (34 if quant == Q8_0 else 18) if quant in (Q8_0, Q4_0) else hd * 2


@dataclass(frozen=True)
class Shape:
    """Geometry of a call: head dim, KV heads, query rows per KV head, quantisation, row stride and head bytes."""
    hd: int
    nkv: int
    rows: int
    quant: int
    rs: int
    hb: int

    def c(self) -> _Shape:
        return _Shape(self.hd, self.nkv, self.rows, self.quant, self.rs, self.hb)


def shape_for(hd: int, nkv: int, rows: int, quant: int = Q8_0, rs: int | None = None) -> Shape:
    hb = head_bytes(quant, hd)
    return Shape(hd, nkv, rows, quant, rs if rs is not None else nkv * hb, hb)


@dataclass
class Seg:
    """nk consecutive key positions at device pointers k, v, folded into output set `set`."""
    k: int
    v: int
    nk: int
    set: int = 0


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream_ptr(stream) -> int:
    """cudaStream_t handle for a torch stream (None: torch's current stream). torch's default stream has handle 0,
    which the C ABI reads as "the context's own stream", so it is passed as cudaStreamLegacy (1) instead."""
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    h = int(getattr(stream, "cuda_stream", stream))
    return h if h != 0 else 1


class Context:
    """A libpacuda context on one device (pa_cuda_create)."""

    def __init__(self, device: int = 0):
        self._h = _P()
        rc = lib().pa_cuda_create(device, ctypes.byref(self._h))
        if rc != OK:
            raise PaCudaError(rc, f"pa_cuda_create(device={device}) failed")
        self.device = device

    @property
    def handle(self):
        return self._h

    def check(self, rc: int, what: str = ""):
        if rc != OK:
            msg = lib().pa_cuda_last_error(self._h).decode(errors="replace")
            raise PaCudaError(rc, f"{what}: {msg}" if what else msg)

    def status(self, stream=None):
        """Synchronise the stream and raise if a kernel gave up a bounded wait (pa_cuda_status)."""
        self.check(lib().pa_cuda_status(self._h, _stream_ptr(stream)), "status")

    def set_timeout_ns(self, ns: int):
        lib().pa_cuda_set_timeout_ns(self._h, int(ns))

    def set_kernel(self, which: int):
        """0: by shape; 1: split-K mma.sync kernel; 2: tcgen05 kernel on single CTAs; 3: tcgen05 kernel on CTA pairs
        (2 and 3: hd 128, quantised rows) — for plans created afterwards."""
        lib().pa_cuda_set_kernel(self._h, int(which))

    def set_qk_domain(self, domain: int):
        """QK_F16 (default) or QK_INT8: the reference's int8-domain QK (Q quantised per 32-block by the Q8_0 rule,
        int32 block dot products with the Q8_0 K bytes, scores in fp32), Q8_0 rows on the split-K kernel only — for
        plans created afterwards."""
        lib().pa_cuda_set_qk_domain(self._h, int(domain))

    def set_stall_test(self, on: bool):
        """Failure-detection hook: the next decode kernels wait on a barrier nothing completes (bounded)."""
        lib().pa_cuda_set_stall_test(self._h, 1 if on else 0)

    @property
    def launches(self) -> int:
        return int(lib().pa_cuda_launch_count(self._h))

    # exchange of the position-shard call (shard_attn_allgather_merge) for calls made afterwards
    EXCHANGE_AUTO, EXCHANGE_ALLGATHER, EXCHANGE_ALLREDUCE, EXCHANGE_PEER = 0, 1, 2, 3

    def set_shard_exchange(self, mode: int):
        """0: by size; 1: all-gather of every rank's packed (O, m, l) and the fold; 2: max / sum all-reduces; 3: peer
        stores over NVLink."""
        lib().pa_cuda_set_shard_exchange(self._h, int(mode))

    def shard_last(self):
        """(exchange, set groups) the last shard call of this context used."""
        e, g = ctypes.c_int(), ctypes.c_int()
        lib().pa_cuda_shard_last(self._h, ctypes.byref(e), ctypes.byref(g))
        return int(e.value), int(g.value)

    def set_shard_groups(self, groups: int):
        """Output-set groups whose exchange overlaps the next group's kernels (0: by size, 1: none)."""
        lib().pa_cuda_set_shard_groups(self._h, int(groups))

    def set_shard_timeout_ms(self, ms: int):
        """> 0: the shard call waits for its exchange and aborts the communicator past ms (raises ETIMEOUT)."""
        lib().pa_cuda_set_shard_timeout_ms(self._h, int(ms))

    def close(self):
        if self._h:
            lib().pa_cuda_destroy(self._h)
            self._h = _P()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


class Plan:
    """The split of a call (output sets x key segments) into chunk jobs, built once, run many times
    (pa_cuda_plan_create / pa_cuda_plan_run)."""

    def __init__(self, ctx: Context, shape: Shape, n_sets: int, segs: Sequence[Seg], chunk_keys: int = 0):
        self.ctx, self.shape, self.n_sets = ctx, shape, n_sets
        arr = (_Seg * max(1, len(segs)))(*[_Seg(s.k, s.v, s.nk, s.set) for s in segs])
        self._h = _P()
        self._sh = shape.c()
        ctx.check(lib().pa_cuda_plan_create(ctx.handle, ctypes.byref(self._sh), n_sets, arr, len(segs), chunk_keys,
                                            ctypes.byref(self._h)), "plan_create")

    @property
    def scratch_bytes(self) -> int:
        return int(lib().pa_cuda_plan_scratch_bytes(self._h))

    @property
    def jobs(self) -> int:
        return int(lib().pa_cuda_plan_jobs(self._h))

    @property
    def launches(self) -> int:
        return int(lib().pa_cuda_plan_launches(self._h))

    @property
    def kernel(self) -> str:
        """Name of the attention-kernel instance the plan launches."""
        return lib().pa_cuda_plan_kernel(self._h).decode()

    def run(self, Qs, O, m, l, stream=None):
        self.ctx.check(lib().pa_cuda_plan_run(self._h, _ptr(Qs), _ptr(O), _ptr(m), _ptr(l), _stream_ptr(stream)),
                       "plan_run")

    def run_host(self, Qs_host, O_host, m_host, l_host, stream=None):
        """Host buffers in, host buffers out (copies inside; returns when they have landed)."""
        self.ctx.check(lib().pa_cuda_plan_run_host(self._h, _ptr(Qs_host), _ptr(O_host), _ptr(m_host), _ptr(l_host),
                                                   _stream_ptr(stream)), "plan_run_host")

    def profile(self, max_runs: int):
        """Record CUDA events around the decode kernel of the next max_runs runs (0: off)."""
        self.ctx.check(lib().pa_cuda_plan_profile(self._h, max_runs), "plan_profile")

    def kernel_ms(self):
        """(summed decode-kernel milliseconds, runs) since profile() / the last call."""
        t = ctypes.c_double()
        n = ctypes.c_uint32()
        self.ctx.check(lib().pa_cuda_plan_kernel_ms(self._h, ctypes.byref(t), ctypes.byref(n)), "plan_kernel_ms")
        return float(t.value), int(n.value)

    def close(self):
        if self._h:
            lib().pa_cuda_plan_destroy(self._h)
            self._h = _P()

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass


def _outputs(shape: Shape, n_sets: int, device):
    import torch
    rows = n_sets * shape.nkv * shape.rows
    O = torch.empty((n_sets, shape.nkv, shape.rows, shape.hd), dtype=torch.float32, device=device)
    m = torch.empty((n_sets, shape.nkv, shape.rows), dtype=torch.float32, device=device)
    l = torch.empty_like(m)
    assert O.numel() == rows * shape.hd
    return O, m, l


def attn(ctx: Context, shape: Shape, Qs, segs: Sequence[Seg], n_sets: int = 1, out=None, stream=None):
    """Partial attention of n_sets output sets over key segments (pa_cuda_attn). Qs: f16 (as int16/float16 tensor)
    [n_sets][nkv][rows][hd] = f16(q*scale). Returns (O, m, l) fp32."""
    O, m, l = out if out is not None else _outputs(shape, n_sets, Qs.device)
    arr = (_Seg * max(1, len(segs)))(*[_Seg(s.k, s.v, s.nk, s.set) for s in segs])
    sh = shape.c()
    ctx.check(lib().pa_cuda_attn(ctx.handle, ctypes.byref(sh), _ptr(Qs), n_sets, arr, len(segs), _ptr(O), _ptr(m),
                                 _ptr(l), _stream_ptr(stream)), "attn")
    return O, m, l


def attn_partial(ctx: Context, shape: Shape, Q, scale: float, K, V, nk: int, stream=None):
    """sme_attn_partial over all heads of one segment: Q fp32 [nkv][rows][hd] unscaled, K/V uint8 rows."""
    O, m, l = _outputs(shape, 1, Q.device)
    sh = shape.c()
    ctx.check(lib().pa_cuda_attn_partial(ctx.handle, ctypes.byref(sh), _ptr(Q), float(scale), _ptr(K), _ptr(V), nk,
                                         _ptr(O), _ptr(m), _ptr(l), _stream_ptr(stream)), "attn_partial")
    return O[0], m[0], l[0]


def merge(ctx: Context, hd: int, Op, mp, lp, out=None, fold: bool = False, stream=None):
    """LSE merge of n partials Op [n][rows][hd], mp/lp [n][rows] -> (O [rows][hd], m, l) (pa_cuda_merge)."""
    import torch
    n = Op.shape[0]
    rows = mp[0].numel() if n else (out[1].numel() if out is not None else 0)
    if out is None:
        O = torch.empty((rows, hd), dtype=torch.float32, device=Op.device)
        m = torch.empty((rows,), dtype=torch.float32, device=Op.device)
        l = torch.empty_like(m)
    else:
        O, m, l = out
    ctx.check(lib().pa_cuda_merge(ctx.handle, hd, rows, n, _ptr(Op), _ptr(mp), _ptr(lp), _ptr(O), _ptr(m), _ptr(l),
                                  1 if fold else 0, _stream_ptr(stream)), "merge")
    return O, m, l


def merge_gathered(ctx: Context, hd: int, rows: int, packed, n_parts: int, out=None, fold: bool = False, stream=None):
    """Merge n_parts partials packed as [n_parts][rows*hd + 2*rows] (O, then m, then l, per part), as one all-gather
    of each rank's packed partial delivers them (pa_cuda_merge_gathered). Returns (O [rows][hd], m, l)."""
    import torch
    if out is None:
        O = torch.empty((rows, hd), dtype=torch.float32, device=packed.device)
        m = torch.empty((rows,), dtype=torch.float32, device=packed.device)
        l = torch.empty_like(m)
    else:
        O, m, l = out
    ctx.check(lib().pa_cuda_merge_gathered(ctx.handle, hd, rows, n_parts, _ptr(packed), _ptr(O), _ptr(m), _ptr(l),
                                           1 if fold else 0, _stream_ptr(stream)), "merge_gathered")
    return O, m, l


def packed_views(buf, rows: int, hd: int):
    """(O, m, l) views into one packed partial buffer of rows*(hd+2) floats."""
    return buf[:rows * hd].view(rows, hd), buf[rows * hd:rows * hd + rows], buf[rows * hd + rows:rows * (hd + 2)]


def normalize(ctx: Context, hd: int, O, m, l, stream=None):
    """O/l -> f16, lse = m + log l (pa_cuda_normalize). Returns (Oh float16, lse fp32)."""
    import torch
    rows = m.numel()
    Oh = torch.empty((rows, hd), dtype=torch.float16, device=O.device)
    lse = torch.empty((rows,), dtype=torch.float32, device=O.device)
    ctx.check(lib().pa_cuda_normalize(ctx.handle, hd, rows, _ptr(O), _ptr(m), _ptr(l), _ptr(Oh), _ptr(lse),
                                      _stream_ptr(stream)), "normalize")
    return Oh, lse


def fold_reply(ctx: Context, hd: int, Oh, lse, O, m, l, stream=None):
    """Fold a normalised reply (f16 Oh [rows][hd], lse [rows]) into the unnormalised partial (O, m, l) in place, as
    the co-attention slot O_unnorm = Oh, l = 1, m = lse (pa_cuda_fold_reply)."""
    rows = lse.numel()
    ctx.check(lib().pa_cuda_fold_reply(ctx.handle, hd, rows, _ptr(Oh), _ptr(lse), _ptr(O), _ptr(m), _ptr(l),
                                       _stream_ptr(stream)), "fold_reply")
    return O, m, l


def nccl_unique_id() -> bytes:
    """The NCCL unique id (128 bytes) one rank creates and every rank passes to NcclComm (pa_cuda_nccl_unique_id)."""
    buf = ctypes.create_string_buffer(128)
    rc = lib().pa_cuda_nccl_unique_id(buf, 128)
    if rc != OK:
        raise PaCudaError(rc, "pa_cuda_nccl_unique_id: NCCL could not be opened or failed")
    return buf.raw


class NcclComm:
    """A communicator of the position-shard ranks over the context's device (pa_cuda_nccl_comm_create)."""

    def __init__(self, ctx: Context, uid: bytes, rank: int, world: int):
        self.ctx = ctx
        h = ctypes.c_void_p()
        idbuf = ctypes.create_string_buffer(bytes(uid), 128)
        ctx.check(lib().pa_cuda_nccl_comm_create(ctx.handle, idbuf, int(rank), int(world), ctypes.byref(h)),
                  "nccl_comm_create")
        self._h = h

    @property
    def handle(self):
        return self._h

    def close(self):
        if self._h:
            lib().pa_cuda_nccl_comm_destroy(self._h)
            self._h = None


def nccl_wait(ctx: Context, comm: NcclComm, stream=None, timeout_ms: int = 0):
    """Wait for the stream's work, aborting the communicator on an NCCL error or after timeout_ms (pa_cuda_nccl_wait)."""
    ctx.check(lib().pa_cuda_nccl_wait(ctx.handle, comm.handle, _stream_ptr(stream), int(timeout_ms)), "nccl_wait")


def shard_attn_allgather_merge(plan: Plan, Qs, comm: NcclComm, O, m, l, stream=None):
    """This rank's plan, one NCCL all-gather of every rank's packed (O, m, l), and their log-sum-exp fold into O, m, l
    (the same on every rank); pa_cuda_shard_attn_allgather_merge."""
    plan.ctx.check(lib().pa_cuda_shard_attn_allgather_merge(plan._h, _ptr(Qs), comm.handle, _ptr(O), _ptr(m), _ptr(l),
                                                            _stream_ptr(stream)), "shard_attn_allgather_merge")
    return O, m, l


def scale_q(ctx: Context, Q, scale: float, stream=None):
    """f16(Q * scale) on the device (pa_cuda_scale_q)."""
    import torch
    Qs = torch.empty(Q.shape, dtype=torch.float16, device=Q.device)
    ctx.check(lib().pa_cuda_scale_q(ctx.handle, _ptr(Q), float(scale), Q.numel(), _ptr(Qs), _stream_ptr(stream)),
              "scale_q")
    return Qs


class Engine:
    """pa::engine over libpacuda (phone-attn/phone-attn.h:166-183): engine-owned pages (host-writable, device-
    resident managed memory), begin() with host f16 Q [ng][nkv][48][hd], end() with host O/m/l."""

    NR = 48

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self._pages = []

    def alloc_page(self, nbytes: int) -> _Page:
        p = _Page()
        self.ctx.check(lib().pa_cuda_alloc_page(self.ctx.handle, nbytes, ctypes.byref(p)), "alloc_page")
        self._pages.append(p)
        return p

    def free_page(self, p: _Page):
        lib().pa_cuda_free_page(self.ctx.handle, ctypes.byref(p))

    @staticmethod
    def page_view(p: _Page, nbytes: int, which: str = "k"):
        """A writable host view (numpy uint8) of a page's K or V memory."""
        import numpy as np
        addr = p.k if which == "k" else p.v
        return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(addr))

    def begin(self, pages: Sequence[_Page], nkeys: Sequence[int], Qs_host, shape: Shape, ng: int = 1, ntok: int = 8):
        arr = (_Page * max(1, len(pages)))(*pages)
        nk = (ctypes.c_uint32 * max(1, len(nkeys)))(*nkeys)
        sh = shape.c()
        self.ctx.check(lib().pa_cuda_begin(self.ctx.handle, arr, nk, len(pages), Qs_host.ctypes.data, ctypes.byref(sh),
                                           ng, ntok), "begin")

    def end(self, O, m, l) -> float:
        ms = lib().pa_cuda_end(self.ctx.handle, O.ctypes.data, m.ctypes.data, l.ctypes.data)
        if ms < 0:
            msg = lib().pa_cuda_last_error(self.ctx.handle).decode(errors="replace")
            raise PaCudaError(ETIMEOUT, f"end: {msg}")
        return ms

    def arm(self, pages: Sequence[_Page], nkeys: Sequence[int], shape: Shape, ntok: int = 8):
        """engine::arm: prepare the likely next one-group call (its plan and a CUDA graph of the whole call)."""
        arr = (_Page * max(1, len(pages)))(*pages)
        nk = (ctypes.c_uint32 * max(1, len(nkeys)))(*nkeys)
        sh = shape.c()
        self.ctx.check(lib().pa_cuda_arm(self.ctx.handle, arr, nk, len(pages), ctypes.byref(sh), ntok), "arm")

    @property
    def graph_calls(self) -> int:
        """begin calls served by an armed graph"""
        return int(lib().pa_cuda_graph_calls(self.ctx.handle))

    @property
    def exec_ms(self) -> float:
        return float(lib().pa_cuda_exec_ms(self.ctx.handle))
