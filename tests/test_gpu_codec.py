"""GPU codec parity: libnsnkv.so against the reference's golden vectors and the oracle.

Bit-exact bar: packed codes, fp16 norm/min/scale, headers and reconstructions
must equal the reference's bytes.
"""
import numpy as np
import pytest
import torch

import golden_util as G
from oracle import nsn_oracle as O

pytestmark = pytest.mark.gpu


def to_dev(x_f32, dtype):
    t = torch.from_numpy(np.ascontiguousarray(x_f32, dtype=np.float32))
    return t.to(getattr(torch, dtype)).cuda()


def layout_like(name, x):
    """Recreate the reference's memory layout (the strided fixtures are transposed views)."""
    e = G.index()["encode"][name]
    if e["channel_stride"] != 1:
        return x.transpose(-1, -2).contiguous().transpose(-1, -2)
    return x


def bits16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("name", sorted(G.index()["encode"]))
def test_encode_decode_matches_reference(name):
    from nsn_b200 import primitives as P
    from nsn_b200 import core
    x32, strided, entry = G.encode_input(name)
    x = layout_like(name, to_dev(x32, entry["dtype"]))
    assert (x.stride(-1) != 1) == strided
    for bits, rec in entry["bits"].items():
        bits = int(bits)
        if "raises" in rec:
            with pytest.raises(P.NumericalFailure):
                P.nsn_encode(x, bits)
            continue
        r = P.encode_blocks(x, bits, packed=True, unpacked=True)
        key = rec["key"]
        packed = r["codes"].reshape(-1).cpu().numpy()
        assert G.matches(key + "_packed", packed), (name, bits)
        for tag, t in zip("nms", r["metas"]):
            assert G.matches(f"{key}_{tag}", bits16(t)), (name, bits, tag)
        q, metas = P.nsn_encode(x, bits)
        assert torch.equal(q, r["q"])
        for dt in ("float16", "bfloat16", "float32"):
            if rec.get("dec_" + dt) is not True:
                continue
            y = P.nsn_decode(q, metas, getattr(torch, dt))
            yb = y.contiguous().view(torch.int32).cpu().numpy().view(np.uint32) if dt == "float32" else bits16(y)
            assert G.matches(f"{key}_dec_{dt}", yb), (name, bits, dt)
        if bits == 3:
            y = core.nsn_int3_qdq(x)
            yb = y.contiguous().view(torch.int32).cpu().numpy().view(np.uint32) if y.dtype == torch.float32 else bits16(y)
            assert G.matches(f"{key}_int3_qdq", yb), name


def test_pack_kats_and_byte_pairs():
    from nsn_b200 import primitives as P
    from nsn_b200 import codec as C
    for case in G.index()["pack_codes"]["cases"]:
        codes = G.get(case["key"] + "_codes")
        want = G.get(case["key"] + "_bytes")
        assert P.pack_codes(codes, case["bits"]) == want.tobytes()
        assert np.array_equal(P.unpack_codes(want.tobytes(), case["count"], case["bits"]), codes)
    for case in G.index()["pack3"]["cases"]:
        n = case["n"]
        a = torch.from_numpy(((np.arange(n) * 5 + 3) % 8).astype(np.uint8)).cuda()
        p = C.pack3(a)
        assert p.cpu().numpy().tobytes() == G.get(case["key"]).tobytes()
        assert torch.equal(C.unpack3(p, (n,)), a)
    a = np.repeat(np.arange(256, dtype=np.uint8), 256)
    b = np.tile(np.arange(256, dtype=np.uint8), 256)
    payload = torch.from_numpy(np.stack((a, b, a ^ b), -1).reshape(-1).copy()).cuda()
    before = payload.clone()
    codes = C.unpack3(payload, (65536 * 8,))
    import hashlib
    assert hashlib.sha256(codes.cpu().numpy().tobytes()).hexdigest() == G.index()["byte_pairs"]["codes_sha256"]
    assert torch.equal(payload, before)
    with pytest.raises(P.ContractError):
        P.pack_codes(np.array([8], np.uint8), 3)


def test_group_codec_cfg0():
    from nsn_b200 import workloads
    from nsn_b200 import codec as C
    k, v, _, _, _ = workloads.np_config(0)
    for name, src in (("cfg0_k", k), ("cfg0_v", v)):
        x = torch.from_numpy(src).cuda().reshape(1, 8, 16, 64, 128)
        g = C.encode_group(x, 0)
        assert G.matches(f"group_{name}_codes", g["codes"].cpu().numpy())
        assert G.matches(f"group_{name}_headers", g["headers"].cpu().numpy())
        for tag, t in zip("nms", g["metas"]):
            assert G.matches(f"group_{name}_{tag}", bits16(t))
        for dt in ("float16", "bfloat16"):
            y = C.restore_group(g, getattr(torch, dt))
            assert G.matches(f"group_{name}_restore_{dt}", bits16(y))
        g2 = C.encode_group(x[:, :, :5], 320)
        assert G.matches(f"group_{name}_headers_start320", g2["headers"].cpu().numpy())
        gg = C.append_group(C.encode_group(x[:, :, :7], 0), C.encode_group(x[:, :, 7:], 7 * 64))
        assert torch.equal(gg["codes"], g["codes"]) and torch.equal(gg["headers"], g["headers"])


def test_full_size_encode_matches_oracle():
    """cfg1-sized K (8 heads x 511 blocks, fp16): every code byte and fp16 metadata equal to the oracle."""
    from nsn_b200 import primitives as P
    from nsn_b200 import workloads
    gen = torch.Generator(device="cuda").manual_seed(1)
    x = workloads.torch_kv(gen, (1, 8, 511 * 64, 128), workloads.K_OUTLIERS_4, 0.5).reshape(1, 8, 511, 64, 128)
    r = P.encode_blocks(x, 3)
    q, n, m, s, st = O.nsn_encode(x.float().cpu().numpy(), 3)
    assert st == 0
    got = r["codes"].cpu().numpy().reshape(-1, 3072)
    want = np.stack([O.pack3(blk) for blk in q.reshape(-1, 64, 128)])
    assert np.array_equal(got, want)
    for t, ref in zip(r["metas"], (n, m, s)):
        assert np.array_equal(bits16(t).reshape(-1), ref.view(np.uint16).reshape(-1))


def test_int5_round_trip_and_restore_against_oracle():
    """INT5 (cfg4 width): encode -> restore equals the oracle's nsn_qdq bit for bit."""
    from nsn_b200 import primitives as P
    from nsn_b200 import workloads
    gen = torch.Generator(device="cuda").manual_seed(4)
    x = workloads.torch_kv(gen, (2, 37, 64, 128), (), 1.0)
    r = P.encode_blocks(x, 5)
    y = P.restore_blocks(r["codes"], r["metas"], torch.float16, bits=5)
    want = O.nsn_qdq(x.float().cpu().numpy(), 5, "float16")
    assert np.array_equal(bits16(y).reshape(-1), want.view(np.uint16).reshape(-1))
    back = P.unpack_codes(r["codes"].reshape(-1), 2 * 37 * 8192, 5)
    q, _ = P.nsn_encode(x, 5)
    assert torch.equal(back, q.reshape(-1))


def _fp16_stress_blocks(rng, n):
    """fp16 blocks [n, 64, 128] from six families that reach the encoder's corners."""
    fam = []
    # heavy-tailed tokens with outlier channels
    x = rng.standard_normal((n, 64, 128)).astype(np.float32) * rng.lognormal(0, 2.0, (n, 64, 1)).astype(np.float32)
    x[..., ::17] *= 50
    fam.append(np.clip(x, -4000, 4000))
    # random finite fp16 bit patterns: every exponent, subnormals, +-0
    b = rng.integers(0, 1 << 16, (n, 64, 128), dtype=np.uint32).astype(np.uint16)
    b[(b & 0x7C00) == 0x7C00] &= 0xBBFF
    fam.append(b.view(np.float16).astype(np.float32))
    # sparse rows: mostly exact zeros of both signs
    x = rng.standard_normal((n, 64, 128)).astype(np.float32)
    x[rng.random((n, 64, 128)) < 0.95] = 0.0
    x[rng.random((n, 64, 128)) < 0.3] *= -1.0
    x[(x == 0) & (rng.random((n, 64, 128)) < 0.5)] = -0.0
    fam.append(x)
    # constant channels and constant tokens
    x = rng.standard_normal((n, 64, 128)).astype(np.float32)
    x[:, :, ::3] = x[:, :1, ::3]
    x[:, ::5, :] = 0.25
    fam.append(x)
    # subnormal-only magnitudes
    x = (rng.integers(-1023, 1024, (n, 64, 128)) * 2.0 ** -24).astype(np.float32)
    fam.append(x)
    # near the fp16 maximum (norms overflow fp16: the status word must say so)
    x = rng.uniform(-65504, 65504, (n, 64, 128)).astype(np.float32)
    fam.append(x)
    return [f.astype(np.float16) for f in fam]


@pytest.mark.parametrize("bits", [3, 4, 5])
def test_fp16_encoder_stress_matches_oracle(bits):
    """The fp16 encoder (reciprocal + quotient correction) equals the oracle bit for bit
    on 6 x 384 blocks per width: codes, packed bytes, fp16 metadata and status."""
    from nsn_b200 import primitives as P
    rng = np.random.default_rng(100 + bits)
    for fi, x16 in enumerate(_fp16_stress_blocks(rng, 384)):
        x = torch.from_numpy(x16).cuda().reshape(3, 128, 64, 128)
        r = P.encode_blocks(x, bits, packed=True, unpacked=True, check=False)
        q, n, m, s, st = O.nsn_encode(x16.astype(np.float32).reshape(3, 128, 64, 128), bits)
        assert int(r["status"].item()) == st, (fi, int(r["status"].item()), st)
        assert np.array_equal(r["q"].cpu().numpy(), q), fi
        for t, ref in zip(r["metas"], (n, m, s)):
            assert np.array_equal(bits16(t).reshape(-1), ref.view(np.uint16).reshape(-1)), fi
        want = np.frombuffer(O.pack_codes(q, bits), np.uint8)
        assert np.array_equal(r["codes"].cpu().numpy().reshape(-1), want), fi
