"""Structural checks of the decode-attention inputs (host side, no device work).

Mirrors experiments/nb06/source/loop_kv_nb06_checks.py:55-71 and
experiments/ac08/source/loop_kv_vf01_checks.py:5-12, generalised from the
hard-coded 48:8 / 16-head shapes to any hq = G*h with G in {1, 2, 4, 6, 8},
fp16 or bf16 tails and query, and INT3/INT4/INT5 groups.

The reference's separate finite scan (loop_kv_vf01_checks.py:20-63, one Triton
launch plus a blocking host read before attention) is not a separate pass
here: the fused kernel checks every q, tail and metadata value it reads and
reports NaN/Inf through its device status word (NSNKV_ST_INPUT_NONFINITE).
"""
from __future__ import annotations

import torch

from . import primitives as w

GROUPS = (1, 2, 4, 6, 8)


def group_layout(group, h, dev):
    """Validate one packed group; return (sealed tokens, bits)."""
    if group is None:
        return 0, None
    codes = group["codes"]
    w.require(codes.dtype == torch.uint8 and codes.ndim == 4 and tuple(codes.shape[:2]) == (1, h)
              and codes.shape[2] > 0, "Codes layout")
    cb = codes.shape[-1]
    w.require(cb in (w.code_bytes(3), w.code_bytes(4), w.code_bytes(5)), "Codes layout")
    bits = cb * 8 // (w.BLOCK * w.DIM)
    n = codes.shape[2]
    w.require(len(group["metas"]) == 3, "Metadata count")
    specs = [(codes, (1, h, n, cb), torch.uint8)]
    if group.get("headers") is not None:
        specs.append((group["headers"], (1, h, n, 12), torch.uint8))
    specs.extend(zip(group["metas"], [(1, h, n, 64, 1), (1, h, n, 1, 128), (1, h, n, 1, 128)], [torch.float16] * 3))
    for x, shape, dtype in specs:
        w.require(tuple(x.shape) == shape and x.dtype == dtype and x.device == dev, "Packed tensor layout/device")
    head_stride_blocks(group)
    return n * 64, bits


def head_stride_blocks(group) -> int:
    """Blocks between one head's first block and the next head's in every tensor of a group.

    A group from encode_group is contiguous (n); PackedCache serves views of arrays with
    spare capacity (the capacity).  Each block must be dense and the blocks of a head
    consecutive, with the same head stride in every tensor of the group.
    """
    tensors = [group["codes"], *group["metas"]] + ([group["headers"]] if group.get("headers") is not None else [])
    strides = set()
    for x in tensors:
        per = 1
        for d in x.shape[3:]:
            per *= d
        inner = x[0, 0, 0] if x.shape[2] else None
        dense_block = inner is None or inner.is_contiguous()
        w.require(dense_block and (x.shape[2] <= 1 or x.stride(2) == per) and x.stride(1) % per == 0
                  and x.stride(1) // per >= x.shape[2], "Packed tensor layout/device")
        strides.add(x.stride(1) // per if x.shape[1] > 1 else x.shape[2])
    w.require(len(strides) == 1, "Packed tensor layout/device")
    return strides.pop()


def structural(g, kt, q, vg, vt):
    """Return (total length, hq, h, bits) after validating shapes, dtypes and devices."""
    w.require(q.dtype in (torch.float16, torch.bfloat16) and q.ndim == 4 and q.shape[0] == 1 and q.shape[2] == 1
              and q.shape[3] == 128 and q.is_contiguous() and q.device.type == "cuda", "Q layout/device")
    h = kt.shape[1] if kt.ndim == 4 else -1
    w.require(h > 0 and q.shape[1] % h == 0 and q.shape[1] // h in GROUPS, "Q/KV head grouping")
    dims = []
    bits_seen = set()
    for group, tail in ((g, kt), (vg, vt)):
        w.require(tail.dtype == q.dtype and tail.ndim == 4 and tuple(tail.shape[:2]) == (1, h)
                  and tail.shape[-1] == 128 and tail.device == q.device and tail.is_contiguous(), "Tail layout/device")
        cc, bits = group_layout(group, h, q.device)
        if bits is not None:
            bits_seen.add(bits)
        dims.append((cc, cc + tail.shape[2]))
    w.require(dims[0] == dims[1] and dims[0][1] > 0, "K/V lengths differ")
    w.require(len(bits_seen) <= 1, "K/V code widths differ")
    return dims[0][1], q.shape[1], h, (bits_seen.pop() if bits_seen else 3)


def expected_headers(n, h, bits, start, device):
    """'<QHBB' headers (start + 64 i, 64, bits, 0) of an [1, h, n] group."""
    off = torch.arange(n, dtype=torch.int64) * 64 + start
    b = torch.zeros((n, 12), dtype=torch.uint8)
    for k in range(8):
        b[:, k] = ((off >> (8 * k)) & 0xFF).to(torch.uint8)
    b[:, 8] = 64
    b[:, 9] = 0
    b[:, 10] = bits
    b[:, 11] = 0
    return b.reshape(1, 1, n, 12).expand(1, h, n, 12).to(device)


def headers_ok(group, start=0) -> bool:
    """Device compare of a group's headers against expected_headers (one host sync)."""
    if group is None or group.get("headers") is None:
        return True
    _, h, n, _ = group["codes"].shape
    bits = group["codes"].shape[-1] * 8 // (w.BLOCK * w.DIM)
    return bool(torch.equal(group["headers"], expected_headers(n, h, bits, start, group["codes"].device)))
