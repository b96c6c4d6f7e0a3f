"""``nsn_int3_qdq``: the ten-line NSN INT3 quantize/reconstruct core on the GPU.

Mirrors papers/nsn-integrated/code/nsn_int3_core.py:11-21.  The reference's own
arithmetic is nsn_qdq(x, 3) (identical results, checked by its golden vectors);
here it is the fused encoder kernel followed by the restore kernel.
"""
from .primitives import nsn_qdq


def nsn_int3_qdq(x):
    return nsn_qdq(x, 3)
