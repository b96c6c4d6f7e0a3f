"""Pin the CPU oracle (oracle/nsn_oracle.py) to the reference's own outputs.

The golden vectors were produced by running the reference's torch/NumPy code
(tests/golden/make_golden.py).  Every comparison here is bit-exact except the
attention bridge, which is compared at the parity tolerance.
"""
import numpy as np
import pytest

import golden_util as G
from oracle import nsn_oracle as O


def test_pack_codes_kats():
    for case in G.index()["pack_codes"]["cases"]:
        codes = G.get(case["key"] + "_codes")
        want = G.get(case["key"] + "_bytes")
        got = np.frombuffer(O.pack_codes(codes, case["bits"]), np.uint8)
        assert got.tobytes() == want.tobytes(), case
        assert np.array_equal(O.unpack_codes(want, case["count"], case["bits"]), codes)


def test_pack3_pattern_and_byte_pairs():
    for case in G.index()["pack3"]["cases"]:
        n = case["n"]
        a = ((np.arange(n) * 5 + 3) % 8).astype(np.uint8)
        assert O.pack3(a).tobytes() == G.get(case["key"]).tobytes()
        assert np.array_equal(O.unpack3(G.get(case["key"]), (n,)), a)
    a = np.repeat(np.arange(256, dtype=np.uint8), 256)
    b = np.tile(np.arange(256, dtype=np.uint8), 256)
    payload = np.stack((a, b, a ^ b), -1).reshape(-1)
    import hashlib
    codes = O.unpack3(payload, (65536 * 8,))
    assert hashlib.sha256(codes.tobytes()).hexdigest() == G.index()["byte_pairs"]["codes_sha256"]


def test_planned_bytes_kats():
    for c in G.index()["planned_bytes"]["cases"]:
        assert O.planned_bytes(tuple(c["shape"]), c["compressed"], c["bits"]) == c["want"]
    with pytest.raises(ValueError):
        O.planned_bytes((1, 1, 100, 128), 65, 3)


@pytest.mark.parametrize("name", sorted(G.index()["encode"]))
def test_encode_decode_bit_exact(name):
    x, strided, entry = G.encode_input(name)
    for bits, rec in entry["bits"].items():
        bits = int(bits)
        q, n, m, s, status = O.nsn_encode(x, bits, strided)
        if "raises" in rec:
            assert status != 0, (name, bits)
            continue
        assert status == 0, (name, bits, status)
        key = rec["key"]
        packed = np.frombuffer(O.pack_codes(q, bits), np.uint8)
        assert G.matches(key + "_packed", packed), (name, bits)
        for tag, t in (("n", n), ("m", m), ("s", s)):
            assert G.matches(f"{key}_{tag}", t.view(np.uint16)), (name, bits, tag)
        for dt in ("float16", "bfloat16", "float32"):
            if rec.get("dec_" + dt) is not True:
                continue
            y = O.nsn_decode(q, n, m, s, dt)
            if dt == "float16":
                yb = y.view(np.uint16)
            elif dt == "bfloat16":
                yb = O.bf16_bits(y)
            else:
                yb = y.view(np.uint32)
            assert G.matches(f"{key}_dec_{dt}", yb), (name, bits, dt)
        if bits == 3:
            assert rec["int3_qdq_equals_nsn_qdq"]
            dtype = entry["dtype"]
            y = O.nsn_int3_qdq(x, dtype, strided)
            yb = {"float16": lambda a: a.view(np.uint16), "bfloat16": O.bf16_bits,
                  "float32": lambda a: a.view(np.uint32)}[dtype](y)
            assert G.matches(f"{key}_int3_qdq", yb), name


def test_group_headers():
    for start, key in ((0, "group_cfg0_k_headers"), (320, "group_cfg0_k_headers_start320")):
        h = G.get(key)
        n = h.shape[2]
        want = O.block_headers(start, n, 3, h.shape[1]).reshape(h.shape)
        assert want.tobytes() == h.tobytes()


def test_group_codes_and_restore():
    from nsn_b200 import workloads
    k, v, _, _, _ = workloads.np_config(0)
    for name, src in (("cfg0_k", k), ("cfg0_v", v)):
        x = src.astype(np.float32).reshape(1, 8, 16, 64, 128)
        q, n, m, s, st = O.nsn_encode(x, 3)
        assert st == 0
        codes = np.stack([O.pack3(q[0, h, i]) for h in range(8) for i in range(16)]).reshape(1, 8, 16, 3072)
        assert G.matches(f"group_{name}_codes", codes)
        y16 = O.nsn_decode(q, n, m, s, "float16").reshape(1, 8, 1024, 128)
        assert G.matches(f"group_{name}_restore_float16", y16.view(np.uint16))
        yb = O.nsn_decode(q, n, m, s, "bfloat16").reshape(1, 8, 1024, 128)
        assert G.matches(f"group_{name}_restore_bfloat16", O.bf16_bits(yb))


@pytest.mark.parametrize("name", sorted(G.index()["attention"]))
def test_bridge_attention_oracle(name):
    e = G.index()["attention"][name]
    dt = e["dtype"]
    if name == "cfg0":
        from nsn_b200 import workloads
        k, v, q, nb, t = workloads.np_config(0)
        kin, vin = k.astype(np.float32), v.astype(np.float32)
        assert G.matches("attn_cfg0_k_in", k.view(np.uint16))
    else:
        kin = G.bits_to_float32(G.get(f"attn_{name}_k_in"), dt)
        vin = G.bits_to_float32(G.get(f"attn_{name}_v_in"), dt)
    q = G.bits_to_float32(G.get(f"attn_{name}_q"), dt)
    nb, t, h = e["blocks"], e["tail"], e["h"]
    fulls = []
    for src in (kin, vin):
        if nb:
            sealed = src[:, :, :nb * 64].reshape(1, h, nb, 64, 128)
            qq, n, m, s, st = O.nsn_encode(sealed, 3)
            assert st == 0
            full = O.restore_full(qq, n, m, s, src[:, :, nb * 64:], dt)
        else:
            full = src
        fulls.append(full)
    out, _ = O.bridge_attention(q, fulls[0], fulls[1])
    ref = G.bits_to_float32(G.get(f"attn_{name}_sdpa"), dt).reshape(out.shape)
    fin = G.bits_to_float32(G.get(f"attn_{name}_finish"), "float32").reshape(out.shape)
    ok, err = O.within_tolerance(out, ref, *O.TOLERANCE[dt])
    assert ok, (name, err)
    ok, err = O.within_tolerance(out, fin, rtol=1e-5, atol=1e-5)
    assert ok, (name, err)


# ---------------------------------------------------------------- the timed CPU bridge port
def _golden_attention_inputs(name):
    e = G.index()["attention"][name]
    dt = e["dtype"]
    if name == "cfg0":
        from nsn_b200 import workloads
        k, v, _, _, _ = workloads.np_config(0)
        kin, vin = k.astype(np.float32), v.astype(np.float32)
    else:
        kin = G.bits_to_float32(G.get(f"attn_{name}_k_in"), dt)
        vin = G.bits_to_float32(G.get(f"attn_{name}_v_in"), dt)
    q = G.bits_to_float32(G.get(f"attn_{name}_q"), dt)
    return e, kin.reshape(1, e["h"], -1, 128), vin.reshape(1, e["h"], -1, 128), q.reshape(1, e["hq"], 1, 128)


@pytest.mark.parametrize("name", sorted(G.index()["attention"]))
def test_bridge_port_reproduces_reference_sdpa(name):
    """oracle/bridge_torch.bridge_decode (the timed CPU baseline) gives the reference's
    recorded SDPA output bit for bit, with groups from the port's own encoder."""
    import torch
    from oracle import bridge_torch as B
    e, kin, vin, q = _golden_attention_inputs(name)
    dt = {"float16": torch.float16, "bfloat16": torch.bfloat16}[e["dtype"]]
    nb, h = e["blocks"], e["h"]
    parts = []
    for src in (kin, vin):
        x = torch.from_numpy(src).to(dt)
        codes, metas = B.encode_group(x[:, :, :nb * 64].reshape(1, h, nb, 64, 128))
        parts.append((codes, metas, x[:, :, nb * 64:].contiguous()))
    out = B.bridge_decode(torch.from_numpy(q).to(dt), *parts[0], *parts[1])
    want = G.get(f"attn_{name}_sdpa")
    assert out.contiguous().view(torch.int16).numpy().view(np.uint16).tobytes() == want.tobytes(), name


@pytest.mark.parametrize("name", sorted(G.index()["encode"]))
def test_bridge_port_encoder_bit_exact(name):
    """The port's nsn_encode + pack3 (its seal step) give the reference's recorded codes and metas."""
    import torch
    from oracle import bridge_torch as B
    x, strided, entry = G.encode_input(name)
    rec = entry["bits"].get("3")
    if strided or rec is None or "raises" in rec:
        pytest.skip("channel-strided or rejected input: the port takes contiguous rows")
    dt = {"float16": torch.float16, "bfloat16": torch.bfloat16, "float32": torch.float32}[entry["dtype"]]
    q, metas = B.nsn_encode(torch.from_numpy(x).to(dt), 3)
    assert G.matches(rec["key"] + "_packed", B.pack3(q).numpy())
    for tag, t in zip(("n", "m", "s"), metas):
        assert G.matches(f"{rec['key']}_{tag}", t.contiguous().view(torch.int16).numpy().view(np.uint16)), tag


def test_bridge_sequence_step_and_seal():
    """BridgeSequence.step equals bridge_decode over the history plus the new token, and
    a tail reaching 64 tokens is encoded into one more block."""
    import torch
    from oracle import bridge_torch as B
    from nsn_b200 import workloads
    rng = np.random.default_rng(4)
    h, hq, nb, t = 2, 8, 2, 62
    k = torch.from_numpy(workloads.np_kv(rng, (1, h, nb * 64 + t + 3, 128), workloads.K_OUTLIERS_4, 0.5))
    v = torch.from_numpy(workloads.np_kv(rng, (1, h, nb * 64 + t + 3, 128), (), 0.5))
    kc, km = B.encode_group(k[:, :, :nb * 64].reshape(1, h, nb, 64, 128))
    vc, vm = B.encode_group(v[:, :, :nb * 64].reshape(1, h, nb, 64, 128))
    seq = B.BridgeSequence(kc, km, k[:, :, nb * 64:nb * 64 + t], vc, vm, v[:, :, nb * 64:nb * 64 + t])
    for i in range(3):
        T = nb * 64 + t + i + 1
        q = torch.from_numpy(rng.standard_normal((1, hq, 1, 128)).astype(np.float16))
        kk, vv = k[:, :, T - 1:T], v[:, :, T - 1:T]
        sealed = seq.k[0].shape[2]
        want = B.bridge_decode(q, seq.k[0], seq.k[1], torch.cat((seq.k[2], kk), 2),
                               seq.v[0], seq.v[1], torch.cat((seq.v[2], vv), 2))
        assert torch.equal(seq.step(q, kk, vv), want)
        assert seq.k[0].shape[2] == sealed + (1 if T - 64 * sealed == 64 else 0)
    assert seq.k[0].shape[2] == nb + 1 and seq.k[2].shape[2] == 1
    codes, metas = B.encode_group(k[:, :, nb * 64:(nb + 1) * 64].reshape(1, h, 1, 64, 128))
    assert torch.equal(seq.k[0][:, :, nb:], codes) and all(torch.equal(a[:, :, nb:], b) for a, b in zip(seq.k[1], metas))


# ---------------------------------------------------------------- library INT3 container
def _asym_input(case):
    """float32 values in the input's logical order (a transposed input was recorded through its view)."""
    return G.bits_to_float32(G.get(f"asym_{case['name']}_x"), case["dtype"]).reshape(case["shape"])


@pytest.mark.parametrize("case", G.index()["int3asym"]["cases"], ids=lambda c: c["name"])
def test_oracle_int3asym_matches_reference(case):
    name = case["name"]
    x = _asym_input(case)
    strided = case["channel_stride"] != 1
    idx, n16, m16, s16 = O.int3asym_encode(x) if not strided else _asym_encode_strided(x)
    packed = np.frombuffer(O.pack_codes(idx, 3), np.uint8).reshape(G.get(f"asym_{name}_packed").shape)
    assert np.array_equal(packed, G.get(f"asym_{name}_packed"))
    assert np.array_equal(n16.view(np.uint16).reshape(-1), G.get(f"asym_{name}_norm").reshape(-1))
    assert np.array_equal(m16.view(np.uint16).reshape(-1), G.get(f"asym_{name}_dmin").reshape(-1))
    assert np.array_equal(s16.view(np.uint16).reshape(-1), G.get(f"asym_{name}_dstep").reshape(-1))
    y = O.int3asym_decode(idx, n16, m16, s16)
    assert np.array_equal(y.view(np.uint16).reshape(-1), G.get(f"asym_{name}_y").reshape(-1))


def _asym_encode_strided(x):
    """The oracle's encode with the sequential norm order of a channel-strided input."""
    a = np.asarray(x, np.float32)
    n = np.maximum(O.row_norm(a, strided=True), np.float32(1e-12))[..., None]
    d = (a / n).astype(np.float32)
    d_min = d.min(axis=-2, keepdims=True)
    d_max = d.max(axis=-2, keepdims=True)
    step = (np.maximum(d_max - d_min, np.float32(1e-12)) / np.float32(7)).astype(np.float32)
    idx = np.clip(np.rint((d - d_min) / step), 0, 7).astype(np.uint8)
    return idx, n.astype(np.float16), d_min.astype(np.float16), step.astype(np.float16)


def test_oracle_int3_unsigned_packing_matches_reference():
    codes = G.get("asym_pack_codes").astype(np.uint8)
    want = G.get("asym_pack_bytes")
    got = np.frombuffer(O.pack_codes(codes, 3), np.uint8).reshape(want.shape)
    assert np.array_equal(got, want)


# ---------------------------------------------------------------- K1c batched decode scores
@pytest.mark.parametrize("cell", G.index()["k1c"]["cells"], ids=lambda c: c["key"])
def test_oracle_k1c_store_and_scores_match_reference(cell):
    import hashlib
    import torch
    from oracle import k1c
    model = k1c.MODELS[cell["model"]]
    q, tstore, ref32 = k1c.make_store(model, cell["B"], cell["T"], cell["bits"], cell["recipe"])
    bits = lambda t: t.contiguous().view(torch.int16).numpy().tobytes() if t.dtype != torch.uint8 else t.numpy().tobytes()
    assert hashlib.sha256(bits(q)).hexdigest() == cell["q_sha256"]
    for f, h in cell["store_sha256"].items():
        assert hashlib.sha256(bits(tstore[f])).hexdigest() == h, f
    got = k1c.gate_scores(q, ref32, cell["recipe"], model).numpy()
    want = G.get(cell["key"] + "_scores")
    assert np.abs(got - want).max() <= 1e-6 * np.abs(want).max()
