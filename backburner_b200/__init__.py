"""backburner_b200 - B200 (sm_100a) engine for Backburner's phone-attn hot path.

Partial attention over an offloaded, position-contiguous segment of a Q8_0 / Q4_0 KV cache, returning the
unnormalised partial (O, m, l) that the host merges with its own by log-sum-exp. The compute runs in
libpacuda.so (hand-written CUDA for sm_100a, C ABI in include/pa_cuda.h); this package is the Python host side
over that ABI (ctypes), mirroring the reference's engine and kernel interfaces:

    sme_attn_partial (scripts/sme/sme_attn.c:271-306)   -> attn_partial()
    sme_attn_pipe / the engine's page batching           -> Plan, attn()
    merge_partial / pa_merge (phone-attn.h:231-239,
        pa-metal.mm:137-159)                             -> merge()
    attn_core's normalisation (phone-attn.h:651-655)     -> normalize()
    the co-attention slot of a reply (phone-attn.h:18-20) -> fold_reply()
    pa::engine (phone-attn.h:166-183)                    -> Engine (pages, begin, end)

There is no CPU fallback: importing works without a GPU (so the host logic can be tested), but every compute call
needs libpacuda.so and a B200; a missing library raises ``LibraryMissing``.
"""
from __future__ import annotations

from .api import (  # noqa: F401
    F16, Q8_0, Q4_0, QK_F16, QK_INT8, PaCudaError, LibraryMissing, Shape, Seg, Context, Plan, Engine, lib, lib_path,
    head_bytes, shape_for, attn, attn_partial, merge, merge_gathered, packed_views, normalize, fold_reply, scale_q,
    available, NcclComm, nccl_unique_id, nccl_wait, shard_attn_allgather_merge,
)
from .formats import quantize_q8_0, quantize_q4_0, dequantize  # noqa: F401
