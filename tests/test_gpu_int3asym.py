"""GPU parity of the library INT3 container against the reference (src/nsn/cache.py, pack.py).

Every field of Int3AsymNsepPchanCache.from_fp16 and every bit of to_fp16 must equal the
values the reference recorded on its own inputs (tests/golden); pack_int3_unsigned must
produce the reference's bytes and reject out-of-range values the same way.
"""
import numpy as np
import pytest
import torch

import golden_util as G

pytestmark = pytest.mark.gpu


def _dtype(name):
    return getattr(torch, name)


def _input(case):
    x = torch.from_numpy(G.bits_to_float32(G.get(f"asym_{case['name']}_x"), case["dtype"]).reshape(case["shape"]))
    x = x.to(_dtype(case["dtype"])).cuda()
    if case["channel_stride"] != 1:  # recreate the reference's transposed view
        x = x.transpose(-1, -2).contiguous().transpose(-1, -2)
    return x


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)


@pytest.mark.parametrize("case", G.index()["int3asym"]["cases"], ids=lambda c: c["name"])
def test_int3asym_matches_reference(case):
    from nsn_b200.cache import Int3AsymNsepPchanCache
    name = case["name"]
    c = Int3AsymNsepPchanCache.from_fp16(_input(case))
    assert np.array_equal(c.packed_d.cpu().numpy(), G.get(f"asym_{name}_packed"))
    assert np.array_equal(_bits(c.norm), G.get(f"asym_{name}_norm").reshape(-1))
    assert np.array_equal(_bits(c.d_min), G.get(f"asym_{name}_dmin").reshape(-1))
    assert np.array_equal(_bits(c.d_step), G.get(f"asym_{name}_dstep").reshape(-1))
    assert c.size_bytes() == case["size_bytes"]
    for y in (c.to_fp16(), c.to_fp16_compiled()):
        assert y.dtype == torch.float16 and tuple(y.shape) == tuple(case["shape"])
        assert np.array_equal(_bits(y), G.get(f"asym_{name}_y").reshape(-1))


def test_int3asym_rejects_what_the_reference_rejects():
    from nsn_b200.cache import Int3AsymNsepPchanCache
    with pytest.raises(AssertionError):
        Int3AsymNsepPchanCache.from_fp16(torch.zeros(1, 4, 12, device="cuda", dtype=torch.float16))
    with pytest.raises(AssertionError):
        Int3AsymNsepPchanCache.from_fp16(torch.zeros(1, 4, 16, device="cuda", dtype=torch.float16), bits=4)


def test_pack_int3_unsigned_matches_reference():
    from nsn_b200.pack import pack_int3_unsigned, unpack_int3_unsigned
    codes = torch.from_numpy(G.get("asym_pack_codes")).to(torch.int8)
    want = G.get("asym_pack_bytes")
    for dev in ("cpu", "cuda"):
        got = pack_int3_unsigned(codes.to(dev))
        assert got.device.type == dev and np.array_equal(got.cpu().numpy(), want)
        back = unpack_int3_unsigned(got, codes.shape[-1])
        assert torch.equal(back.cpu(), codes)
    with pytest.raises(ValueError):
        pack_int3_unsigned(torch.tensor([[0, 1, 2, 3, 4, 5, 6, 8]], dtype=torch.int8))
    clamped = pack_int3_unsigned(torch.tensor([[0, 1, 2, 3, 4, 5, 6, 9]], dtype=torch.int8), strict=False)
    assert torch.equal(unpack_int3_unsigned(clamped, 8), torch.tensor([[0, 1, 2, 3, 4, 5, 6, 7]], dtype=torch.int8))
