"""Sequence-position shards of the offloaded KV across the GPUs of one node (one process per GPU).

Rank r of N holds positions [start, start + count) of every layer: equal shares, the last rank takes the remainder
(the two-phone split of docs/TWO-PHONES.md:14-18, generalised), or explicit uneven shares. Each rank
computes its partial (O, m, l) and packs it as one buffer of rows*(hd+2) floats: O [rows][hd], then m [rows], then l
[rows]; one all-gather of those buffers gives the layout pa_cuda_merge_gathered folds.
"""
from __future__ import annotations

from typing import Sequence


def shard_range(n_keys: int, world: int, rank: int, shares: Sequence[int] | None = None) -> tuple[int, int]:
    """(start, count) of rank `rank`'s positions. shares: explicit per-rank counts summing to n_keys."""
    if shares is not None:
        if len(shares) != world or sum(shares) != n_keys or min(shares) < 0:
            raise ValueError("shares must be world non-negative counts summing to n_keys")
        return sum(shares[:rank]), shares[rank]
    per = n_keys // world
    start = rank * per
    return start, (per if rank < world - 1 else n_keys - start)


def packed_size(rows: int, hd: int) -> int:
    return rows * (hd + 2)


def pack(O, m, l, out=None):
    """Pack (O [rows][hd], m [rows], l [rows]) into one flat buffer (numpy or torch)."""
    rows, hd = O.shape[-2] if O.ndim >= 2 else 1, O.shape[-1]
    rows = m.reshape(-1).shape[0]
    if out is None:
        try:
            import torch
            if isinstance(O, torch.Tensor):
                out = torch.empty(packed_size(rows, hd), dtype=O.dtype, device=O.device)
        except ImportError:
            pass
        if out is None:
            import numpy as np
            out = np.empty(packed_size(rows, hd), dtype=O.dtype)
    out[:rows * hd] = O.reshape(-1)
    out[rows * hd:rows * hd + rows] = m.reshape(-1)
    out[rows * hd + rows:] = l.reshape(-1)
    return out


def unpack(buf, rows: int, hd: int):
    """(O, m, l) views of a packed buffer."""
    return buf[:rows * hd].reshape(rows, hd), buf[rows * hd:rows * hd + rows], buf[rows * hd + rows:rows * (hd + 2)]
