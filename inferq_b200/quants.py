"""GGUF block encoders for synthetic checkpoints (Q4_K, Q5_K, Q6_K, Q8_0).

The reference never quantizes weights itself -- it reads GGUF files written by
llama.cpp (``src/gguf.rs:1234-1253``).  These vectorised torch encoders write
valid blocks of the same on-disk formats so seeded random-init checkpoints can
be produced on the host or directly on the GPU.  They are data generators:
the decoder that matters for parity is the block decode the verify path uses,
pinned against gguf-py in ``tests/test_oracle_formats.py``.

Every encoder maps a float tensor ``[rows, cols]`` to uint8 ``[rows, row_bytes]``.
"""
from __future__ import annotations

import torch

F32, F16, Q8_0, Q4_K, Q5_K, Q6_K, Q8_K, BF16 = 0, 1, 8, 12, 13, 14, 15, 30
BLOCK = {Q8_0: 32, Q4_K: 256, Q5_K: 256, Q6_K: 256, F32: 1, F16: 1, BF16: 1}
BLOCK_BYTES = {Q8_0: 34, Q4_K: 144, Q5_K: 176, Q6_K: 210, F32: 4, F16: 2, BF16: 2}
NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q5_K: "Q5_K", Q6_K: "Q6_K", BF16: "BF16"}


def row_bytes(dtype: int, cols: int) -> int:
    if cols % BLOCK[dtype]:
        raise ValueError(f"{cols} columns is not a multiple of the {NAMES[dtype]} block")
    return cols // BLOCK[dtype] * BLOCK_BYTES[dtype]


def _round_away(v: torch.Tensor) -> torch.Tensor:
    return torch.sign(v) * torch.floor(v.abs() + 0.5)


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """[..] f32 -> [.., 2] uint8 little-endian f16."""
    return v.to(torch.float16).contiguous().view(torch.uint8).reshape(*v.shape, 2)


def _safe_div(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.where(b != 0, a / torch.where(b != 0, b, torch.ones_like(b)), torch.zeros_like(a))


def _pack_k_scales(sc: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """Eight 6-bit scales and mins -> the 12 packed bytes of Q4_K/Q5_K."""
    sc = sc.to(torch.int32)
    mn = mn.to(torch.int32)
    lo = (sc[:, :4] & 63) | ((sc[:, 4:] >> 4) << 6)
    mid = (mn[:, :4] & 63) | ((mn[:, 4:] >> 4) << 6)
    hi = (sc[:, 4:] & 15) | ((mn[:, 4:] & 15) << 4)
    return torch.cat([lo, mid, hi], dim=1).to(torch.uint8)


def _kquant_affine(x: torch.Tensor, levels: int):
    """Shared Q4_K/Q5_K: per-32 (min, scale) quantised against f16 d/dmin."""
    sub = x.reshape(-1, 8, 32)
    mn = torch.clamp(sub.amin(dim=2), max=0.0)
    mx = sub.amax(dim=2)
    scale = (mx - mn) / levels
    mval = -mn
    d = (scale.amax(dim=1) / 63).to(torch.float16).to(torch.float32)
    dmin = (mval.amax(dim=1) / 63).to(torch.float16).to(torch.float32)
    sc = torch.clamp(_round_away(_safe_div(scale, d[:, None])), 0, 63)
    m = torch.clamp(_round_away(_safe_div(mval, dmin[:, None])), 0, 63)
    step = d[:, None] * sc
    q = _round_away(_safe_div(sub + (dmin[:, None] * m)[:, :, None], step[:, :, None].expand_as(sub)))
    q = torch.clamp(q, 0, levels).to(torch.int32).reshape(-1, 256)
    return d, dmin, sc, m, q


def _encode_q4k(x: torch.Tensor) -> torch.Tensor:
    d, dmin, sc, m, q = _kquant_affine(x, 15)
    q = q.reshape(-1, 4, 2, 32)
    qs = (q[:, :, 0, :] | (q[:, :, 1, :] << 4)).reshape(-1, 128).to(torch.uint8)
    return torch.cat([_f16_bytes(d), _f16_bytes(dmin), _pack_k_scales(sc, m), qs], dim=1)


def _encode_q5k(x: torch.Tensor) -> torch.Tensor:
    d, dmin, sc, m, q = _kquant_affine(x, 31)
    low = q & 15
    high = (q >> 4) & 1  # [n, 256]
    hb = high.reshape(-1, 8, 32)
    qh = torch.zeros(hb.shape[0], 32, dtype=torch.int32, device=x.device)
    for s in range(8):
        qh |= hb[:, s, :] << s
    low = low.reshape(-1, 4, 2, 32)
    qs = (low[:, :, 0, :] | (low[:, :, 1, :] << 4)).reshape(-1, 128)
    return torch.cat([_f16_bytes(d), _f16_bytes(dmin), _pack_k_scales(sc, m),
                      qh.to(torch.uint8), qs.to(torch.uint8)], dim=1)


def _encode_q6k(x: torch.Tensor) -> torch.Tensor:
    sub = x.reshape(-1, 16, 16)
    scale = sub.abs().amax(dim=2) / 31
    d = (scale.amax(dim=1) / 127).to(torch.float16).to(torch.float32)
    sc = torch.clamp(_round_away(_safe_div(scale, d[:, None])), 0, 127)
    step = (d[:, None] * sc)[:, :, None].expand_as(sub)
    q = torch.clamp(_round_away(_safe_div(sub, step)), -32, 31).to(torch.int32) + 32
    q = q.reshape(-1, 2, 4, 32)  # [n, half, quarter(l//32), i]
    ql = torch.cat([(q[:, :, 0, :] & 15) | ((q[:, :, 2, :] & 15) << 4),
                    (q[:, :, 1, :] & 15) | ((q[:, :, 3, :] & 15) << 4)], dim=2)
    qh = ((q[:, :, 0, :] >> 4) | ((q[:, :, 1, :] >> 4) << 2)
          | ((q[:, :, 2, :] >> 4) << 4) | ((q[:, :, 3, :] >> 4) << 6))
    return torch.cat([ql.reshape(-1, 128).to(torch.uint8), qh.reshape(-1, 64).to(torch.uint8),
                      sc.to(torch.int8).view(torch.uint8), _f16_bytes(d)], dim=1)


def _encode_q80(x: torch.Tensor) -> torch.Tensor:
    blk = x.reshape(-1, 32)
    d = blk.abs().amax(dim=1) / 127
    inv = _safe_div(torch.ones_like(d), d)
    q = _round_away(blk * inv[:, None]).to(torch.int8).view(torch.uint8)
    return torch.cat([_f16_bytes(d), q], dim=1)


_ENCODERS = {Q4_K: _encode_q4k, Q5_K: _encode_q5k, Q6_K: _encode_q6k, Q8_0: _encode_q80}


def encode(x: torch.Tensor, dtype: int) -> torch.Tensor:
    """Encode ``x`` ([rows, cols], float) as GGUF blocks: uint8 [rows, row_bytes]."""
    rows, cols = x.shape
    rb = row_bytes(dtype, cols)
    x = x.to(torch.float32)
    if dtype == F32:
        return x.contiguous().view(torch.uint8).reshape(rows, rb)
    if dtype == F16:
        return x.to(torch.float16).contiguous().view(torch.uint8).reshape(rows, rb)
    if dtype == BF16:
        return x.to(torch.bfloat16).contiguous().view(torch.uint8).reshape(rows, rb)
    out = _ENCODERS[dtype](x.reshape(-1, BLOCK[dtype]).contiguous())
    return out.reshape(rows, rb).contiguous()
