"""Access to the golden vectors recorded from the reference (tests/golden/make_golden.py)."""
import hashlib
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent / "golden"


@lru_cache(None)
def index():
    return json.loads((HERE / "golden.json").read_text())


@lru_cache(None)
def arrays():
    return dict(np.load(HERE / "golden.npz"))


def has(name):
    return name in arrays() or name in index()["hashed"]


def get(name):
    return arrays()[name]


def matches(name, a) -> bool:
    """True when ``a`` equals the recorded array bit for bit (stored or sha256-pinned)."""
    a = np.ascontiguousarray(a)
    if name in arrays():
        want = arrays()[name]
        return want.shape == a.shape and want.dtype == a.dtype and want.tobytes() == a.tobytes()
    h = index()["hashed"][name]
    return list(a.shape) == h["shape"] and str(a.dtype) == h["dtype"] and hashlib.sha256(a.tobytes()).hexdigest() == h["sha256"]


def bits_to_float32(bits, dtype):
    """Recorded raw bits -> float32 values for dtype in {float16, bfloat16, float32}."""
    bits = np.asarray(bits)
    if dtype == "float16":
        return bits.view(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return (bits.astype(np.uint32) << 16).view(np.float32)
    if dtype == "float32":
        return bits.view(np.float32)
    raise ValueError(dtype)


def encode_input(name):
    """float32 values of a recorded encode input plus whether its channel axis is strided."""
    e = index()["encode"][name]
    if name in ("cfg0_k", "cfg0_v"):
        from nsn_b200 import workloads
        k, v, _, _, _ = workloads.np_config(0)
        x = (k if name == "cfg0_k" else v).reshape(e["shape"])
        assert matches(f"enc_{name}_x", x.view(np.uint16))
        return x.astype(np.float32), e["channel_stride"] != 1, e
    x = bits_to_float32(get(f"enc_{name}_x"), e["dtype"]).reshape(e["shape"])
    return x, e["channel_stride"] != 1, e
