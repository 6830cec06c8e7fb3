"""Q8_0 / Q4_0 block formats as torch ops (device-side generation of the synthetic KV the bench and the full-size
tests use). Byte layout and rounding follow the reference:

  Q8_0 (phone-attn/pa-tool.cpp:22-25): per 32 values d = max|x|/127 stored as f16, q = rint(x / f16(d)) in [-127, 127],
       block = f16 d + 32 int8 (34 bytes).
  Q4_0 (the BASELINE rule; nibble order of phone-attn/pa-metal.mm:302-305): d = max|x|/7 stored as f16,
       n = rint(x / f16(d)) + 8 clamped to [1, 15], byte i = n[i] | n[i+16] << 4, value (n - 8) * d (18 bytes).
A head row of hd values is hd/32 consecutive blocks; a key position is nkv head rows back to back.
"""
from __future__ import annotations


def quantize_q8_0(x):
    """x: float32 [..., hd] (hd a multiple of 32) -> uint8 [..., hd/32*34]."""
    import torch
    *lead, hd = x.shape
    xb = x.reshape(-1, hd // 32, 32).float()
    am = xb.abs().amax(dim=-1)
    d16 = (am / 127).to(torch.float16)
    df = d16.float()
    inv = torch.where(df != 0, 1.0 / df, torch.zeros_like(df))
    q = torch.round(xb * inv.unsqueeze(-1)).clamp_(-127, 127).to(torch.int8)
    out = torch.empty((xb.shape[0], hd // 32, 34), dtype=torch.uint8, device=x.device)
    out[..., :2] = d16.view(torch.uint8).reshape(xb.shape[0], hd // 32, 2)
    out[..., 2:] = q.view(torch.uint8)
    return out.reshape(*lead, hd // 32 * 34)


def quantize_q4_0(x):
    """x: float32 [..., hd] -> uint8 [..., hd/32*18]."""
    import torch
    *lead, hd = x.shape
    xb = x.reshape(-1, hd // 32, 32).float()
    am = xb.abs().amax(dim=-1)
    d16 = (am / 7).to(torch.float16)
    df = d16.float()
    inv = torch.where(df != 0, 1.0 / df, torch.zeros_like(df))
    n = (torch.round(xb * inv.unsqueeze(-1)) + 8).clamp_(1, 15).to(torch.uint8)
    out = torch.empty((xb.shape[0], hd // 32, 18), dtype=torch.uint8, device=x.device)
    out[..., :2] = d16.view(torch.uint8).reshape(xb.shape[0], hd // 32, 2)
    out[..., 2:] = n[..., :16] | (n[..., 16:] << 4)
    return out.reshape(*lead, hd // 32 * 18)


def dequantize(rows, quant: int, hd: int):
    """uint8 [..., hd/32*GB] -> float32 [..., hd], exact (f16 scale times the integer)."""
    import torch
    *lead, nb = rows.shape
    gb = 34 if quant == 1 else 18
    blk = rows.reshape(-1, hd // 32, gb)
    d = blk[..., :2].contiguous().view(torch.float16).float()  # [N, nblk, 1]
    if quant == 1:
        q = blk[..., 2:].contiguous().view(torch.int8).float()
    else:
        b = blk[..., 2:].to(torch.int16)
        q = torch.cat([(b & 15) - 8, (b >> 4) - 8], dim=-1).float()
    return (q * d).reshape(*lead, hd)
