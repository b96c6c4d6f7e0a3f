"""Block codec surface: the reference's codec module on the GPU.

Mirrors experiments/nb06/source/loop_kv_nb06_codec.py (== the codec half of
experiments/ac08/source/loop_kv_pk01_cache.py):

  pack3 / unpack3        :6-26   INT3 3-byte-group pack (same bytes as pack_codes(q, 3))
  encode_group(x, start) :28-34  one fused encoder launch -> codes, fp16 metas, headers
  restore_group(g, dtype):36-38  one restore launch, bit-exact with nsn_decode
  append_group(old, new) :40-45
  tensor_inventory       :47-62
  full_pair              :64-66

A group ``g`` is the reference's dict: codes uint8 [1,H,n,3072], metas =
(norm fp16 [1,H,n,64,1], min fp16 [1,H,n,1,128], scale fp16 [1,H,n,1,128]),
headers uint8 [1,H,n,12] ('<QHBB' token offset, 64, bits, 0).  ``bits`` is 3
unless a group was encoded with another width (the header carries it).
"""
from __future__ import annotations

from collections import Counter

import torch

from . import primitives as w


def pack3(q: torch.Tensor) -> torch.Tensor:
    w.require(q.dtype == torch.uint8, "3bit code range/dtype")
    out = w.pack_codes(q.contiguous().reshape(-1), 3)
    return out


def unpack3(payload: torch.Tensor, shape) -> torch.Tensor:
    n = 1
    for x in shape:
        n *= x
    w.require(payload.dtype == torch.uint8 and payload.numel() == (n * 3 + 7) // 8, "3bit payload shape")
    return w.unpack_codes(payload.reshape(-1), n, 3).reshape(shape).contiguous()


def encode_group(x: torch.Tensor, start: int, bits: int = 3):
    """x is [1,H,nblocks,64,128]; keeps no view into x or into uncompressed codes."""
    w.require(x.ndim == 5 and tuple(x.shape[-2:]) == (w.BLOCK, w.DIM), "NSN block shape")
    r = w.encode_blocks(x, bits, packed=True, headers_start=start)
    return dict(codes=r["codes"], metas=tuple(r["metas"]), headers=r["headers"])


def group_bits(g) -> int:
    return int(g["codes"].shape[-1] * 8 // (w.BLOCK * w.DIM))


def restore_group(g, dtype):
    b, h, n, _ = g["codes"].shape
    y = w.restore_blocks(g["codes"].reshape(b * h, n, -1), tuple(m.reshape(b * h, n, *m.shape[-2:]) for m in g["metas"]),
                         dtype, bits=group_bits(g))
    return y.reshape(b, h, n * w.BLOCK, w.DIM)


def append_group(old, new):
    if old is None:
        return new
    return dict(codes=torch.cat((old["codes"], new["codes"]), 2),
                metas=tuple(torch.cat((a, b), 2) for a, b in zip(old["metas"], new["metas"])),
                headers=torch.cat((old["headers"], new["headers"]), 2))


def tensor_inventory(cache):
    tensors = []
    for kv, data in (("K", cache.key_cache), ("V", cache.value_cache)):
        for slot, x in enumerate(data):
            if x is not None:
                tensors.append(("native_tail" if hasattr(cache, "packed") and cache.bits else "float_kv", x))
            g = getattr(cache, "packed", {}).get((slot, kv))
            if g:
                tensors.extend([("codes", g["codes"]), ("headers", g["headers"])])
                tensors.extend(("metadata", v) for v in g["metas"])
    components = Counter()
    seen = {}
    devices = set()
    for name, t in tensors:
        components[name] += t.numel() * t.element_size()
        st = t.untyped_storage()
        seen[(str(t.device), st.data_ptr())] = st.nbytes()
        devices.add(str(t.device))
    return dict(component_bytes=dict(components), tensor_bytes=sum(components.values()),
                unique_storage_bytes=sum(seen.values()), tensor_count=len(tensors), storage_count=len(seen),
                devices=sorted(devices),
                compressed_tokens=cache.compressed.get(0, 0) if hasattr(cache, "compressed") else 0)


def full_pair(cache, slot):
    if hasattr(cache, "materialize"):
        return cache.materialize(slot, "K"), cache.materialize(slot, "V")
    return cache.key_cache[slot], cache.value_cache[slot]
