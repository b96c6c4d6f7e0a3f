"""INT3 packing of the library API (src/nsn/pack.py:85-163).

``pack_int3_unsigned`` / ``unpack_int3_unsigned`` store 8 indices in [0, 7] per 3 bytes,
LSB first. That is the same bitstream as the block codec's INT3 packing, so the work
runs on ``nsnkv_pack`` / ``nsnkv_unpack``. Inputs may live on the CPU or the GPU, and
results come back on the input's device.
"""
from __future__ import annotations

import torch

from . import _lib as L


def pack_int3_unsigned(x_int8, strict=True):
    *prefix, N = x_int8.shape
    assert N % 8 == 0, f"Last dim must be divisible by 8, got {N}"
    L.require_cuda()
    if strict:
        xmin = int(x_int8.min().item())
        xmax = int(x_int8.max().item())
        if xmin < 0 or xmax > 7:
            raise ValueError(
                f"pack_int3_unsigned requires values in [0, 7] (INT3 unsigned range); got [{xmin}, {xmax}]. "
                f"Pass strict=False to silently clamp.")
    codes = x_int8.to(torch.int64).clamp(0, 7).to(torch.uint8).cuda().contiguous().reshape(-1)
    out = torch.empty((codes.numel() * 3 // 8,), dtype=torch.uint8, device=codes.device)
    status = L.status_tensor(codes.device)
    if codes.numel():
        L.check(L.load().nsnkv_pack(L.ptr(codes), codes.numel(), 3, L.ptr(out), L.ptr(status),
                                    L.stream_handle(codes.device)), "nsnkv_pack")
    return out.view(*prefix, 3 * N // 8).to(x_int8.device)


def unpack_int3_unsigned(bytes_in, N):
    *prefix, P = bytes_in.shape
    assert P == 3 * N // 8, f"Expected {3 * N // 8} bytes for N={N}, got {P}"
    L.require_cuda()
    payload = bytes_in.cuda().contiguous().reshape(-1)
    count = payload.numel() * 8 // 3
    out = torch.empty((count,), dtype=torch.uint8, device=payload.device)
    if count:
        L.check(L.load().nsnkv_unpack(L.ptr(payload), count, 3, L.ptr(out), L.stream_handle(payload.device)),
                "nsnkv_unpack")
    return out.view(*prefix, N).to(torch.int8).to(bytes_in.device)
