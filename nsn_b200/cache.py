"""Library INT3 container: ``Int3AsymNsepPchanCache`` (src/nsn/cache.py:134-313).

A tensor [..., T, D] (D % 8 == 0, D <= 256) is held as:
- per-token fp16 norms;
- per-channel fp16 (d_min, d_step) of the unit directions over all T tokens;
- 3-bit unsigned indices, 8 per 3 bytes.

Field names, shapes, asserts and ``size_bytes`` are the reference's. The arithmetic
runs in libnsnkv.so (``nsnkv_int3asym_encode`` / ``_decode``) and reproduces the
reference's CPU results bit for bit. ``to_fp16_compiled`` is the reference's
torch.compile fast path; here it is the same fused kernel as ``to_fp16``.
"""
from __future__ import annotations

import math

import torch

from . import _lib as L
from .primitives import norm_order_of


class Int3AsymNsepPchanCache:
    """Real-packed INT3 asymmetric nsep+pchan cache (fields as src/nsn/cache.py:152-165)."""

    def __init__(self):
        self.packed_d = None
        self.norm = None
        self.d_min = None
        self.d_step = None

    @classmethod
    def from_fp16(cls, x, bits=3):
        assert bits == 3, f"Int3AsymNsepPchanCache packs 3-bit only; got bits={bits}"
        assert x.shape[-1] % 8 == 0, f"Last dim (head_dim) must be divisible by 8, got {x.shape[-1]}"
        L.require_cuda()
        *prefix, T, D = x.shape
        rows = math.prod(prefix) if prefix else 1
        dev = x.device
        order = norm_order_of(x)
        xc = x.contiguous()
        obj = cls()
        obj.packed_d = torch.empty(tuple(prefix) + (T, 3 * D // 8), dtype=torch.uint8, device=dev)
        obj.norm = torch.empty(tuple(prefix) + (T, 1), dtype=torch.float16, device=dev)
        obj.d_min = torch.empty(tuple(prefix) + (1, D), dtype=torch.float16, device=dev)
        obj.d_step = torch.empty(tuple(prefix) + (1, D), dtype=torch.float16, device=dev)
        lib = L.load()
        need = lib.nsnkv_int3asym_scratch_bytes(rows, T, D)
        scratch = torch.empty((max(need, 4),), dtype=torch.uint8, device=dev)
        status = L.status_tensor(dev)
        L.check(lib.nsnkv_int3asym_encode(L.ptr(xc), L.DTYPE_CODE[x.dtype], rows, T, D, order, L.ptr(obj.packed_d),
                                          L.ptr(obj.norm), L.ptr(obj.d_min), L.ptr(obj.d_step), L.ptr(scratch), need,
                                          L.ptr(status), L.stream_handle(dev)),
                "nsnkv_int3asym_encode")
        return obj

    def to_fp16(self):
        """Reconstruct an approximate FP16 tensor [..., T, D]."""
        L.require_cuda()
        *prefix, T, P = self.packed_d.shape
        D = P * 8 // 3
        rows = math.prod(prefix) if prefix else 1
        dev = self.packed_d.device
        out = torch.empty(tuple(prefix) + (T, D), dtype=torch.float16, device=dev)
        # contiguous copies stay referenced until the launch is enqueued
        packed, norm, d_min, d_step = (t.contiguous() for t in (self.packed_d, self.norm, self.d_min, self.d_step))
        L.check(L.load().nsnkv_int3asym_decode(L.ptr(packed), L.ptr(norm), L.ptr(d_min), L.ptr(d_step), rows,
                                               T, D, L.ptr(out), L.stream_handle(dev)),
                "nsnkv_int3asym_decode")
        return out

    def to_fp16_compiled(self):
        """The reference's compiled fast path; the decode kernel is already one fused launch."""
        return self.to_fp16()

    def size_bytes(self):
        """Total bytes in real storage (packed + norm + d_min + d_step)."""
        return self.packed_d.numel() * 1 + self.norm.numel() * 2 + self.d_min.numel() * 2 + self.d_step.numel() * 2
