"""GPU attention parity: fused packed-KV decode attention against the reference's
bridge (golden SDPA outputs recorded from the reference) and the fp64 oracle.

Tolerance (oracle.TOLERANCE): fp16 outputs within 2e-3 relative + 1e-3 absolute
elementwise; bf16 outputs within 1e-2 + 1e-2 (8 significant bits).
"""
import hashlib

import numpy as np
import pytest
import torch

import golden_util as G
from oracle import nsn_oracle as O

pytestmark = pytest.mark.gpu


def np_f32(t):
    return t.float().cpu().numpy()


def make_case(k, v, q, nb, dtype):
    """Seal the first nb blocks with the GPU encoder; return (g, kt, q, vg, vt) like the reference."""
    from nsn_b200 import codec as C
    dt = getattr(torch, dtype)
    kt = torch.from_numpy(np.ascontiguousarray(k, np.float32)).to(dt).cuda()
    vt = torch.from_numpy(np.ascontiguousarray(v, np.float32)).to(dt).cuda()
    qq = torch.from_numpy(np.ascontiguousarray(q, np.float32)).to(dt).cuda()
    h = kt.shape[1]
    if nb:
        g = C.encode_group(kt[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0)
        vg = C.encode_group(vt[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0)
    else:
        g = vg = None
    return g, kt[:, :, nb * 64:].contiguous(), qq, vg, vt[:, :, nb * 64:].contiguous()


def oracle_out(k, v, q, nb, dtype, bits=3):
    h = k.shape[1]
    fulls = []
    for src in (k, v):
        src = np.asarray(src, np.float32)
        if nb:
            qq, n, m, s, st = O.nsn_encode(src[:, :, :nb * 64].reshape(1, h, nb, 64, 128), bits)
            assert st == 0
            fulls.append(O.restore_full(qq, n, m, s, src[:, :, nb * 64:], dtype))
        else:
            fulls.append(src)
    out, lse = O.bridge_attention(np.asarray(q, np.float32), fulls[0], fulls[1])
    return out, lse


def golden_inputs(name):
    e = G.index()["attention"][name]
    dt = e["dtype"]
    if name == "cfg0":
        from nsn_b200 import workloads
        k, v, q, nb, t = workloads.np_config(0)
        return k.astype(np.float32), v.astype(np.float32), q.astype(np.float32), nb, dt
    k = G.bits_to_float32(G.get(f"attn_{name}_k_in"), dt)
    v = G.bits_to_float32(G.get(f"attn_{name}_v_in"), dt)
    q = G.bits_to_float32(G.get(f"attn_{name}_q"), dt)
    return k, v, q, e["blocks"], dt


@pytest.mark.parametrize("name", sorted(G.index()["attention"]))
@pytest.mark.parametrize("arm", ["V_FUSED", "TILE_MATERIALIZE", "TORCH_SDPA"])
def test_pipeline_matches_reference_bridge(name, arm):
    from nsn_b200 import kernel as K
    k, v, q, nb, dt = golden_inputs(name)
    data = make_case(k, v, q, nb, dt)
    def digest(t):
        return hashlib.sha256(t.contiguous().view(torch.int16).cpu().numpy().tobytes()).hexdigest()

    inputs = [data[1], data[2], data[4]] + ([data[0]["codes"], *data[0]["metas"]] if data[0] else [])
    hashes = [digest(t) if t.dtype != torch.uint8 else hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()
              for t in inputs]
    out = K.pipeline(arm, data)
    assert K.LAST_STAGE == "returned"
    after = [digest(t) if t.dtype != torch.uint8 else hashlib.sha256(t.cpu().numpy().tobytes()).hexdigest()
             for t in inputs]
    assert after == hashes, "inputs were modified"
    got = np_f32(out).reshape(q.shape[1], 128)
    ref = G.bits_to_float32(G.get(f"attn_{name}_sdpa"), dt).reshape(q.shape[1], 128)
    ok, err = O.within_tolerance(got, ref, *O.TOLERANCE[dt])
    assert ok, (name, arm, err)
    want, _ = oracle_out(k, v, q, nb, dt)
    ok, err = O.within_tolerance(got, want[0], *O.TOLERANCE[dt])
    assert ok, (name, arm, err)


def test_fused_context_fp32_is_tight():
    """The fp32 context of the fused kernel is within 5e-5 + 1e-5*|x| of the fp64 oracle (cfg0).

    Both use the same bridge-rounded K/V; the residual is fp32 accumulation in the
    tensor cores and the fp16 hi+lo split of the softmax weights."""
    from nsn_b200 import kernel as K
    k, v, q, nb, dt = golden_inputs("cfg0")
    out, ctx, _, _ = K.launch(*make_case(k, v, q, nb, dt))
    want, _ = oracle_out(k, v, q, nb, dt)
    ok, err = O.within_tolerance(np_f32(ctx).reshape(32, 128), want[0], 1e-5, 5e-5)
    assert ok, err


@pytest.mark.parametrize("dtype", ["float16", "bfloat16"])
def test_cfg1_full_size_fused_vs_bridge(dtype):
    """cfg1: 511 INT3 blocks + 64-token tail, GQA 32:8, q ~ N(0,1)/sqrt(128): fused vs oracle and vs the bridge arms."""
    from nsn_b200 import kernel as K
    from nsn_b200 import workloads
    gen = torch.Generator(device="cuda").manual_seed(1)
    T = 511 * 64 + 64
    k = workloads.torch_kv(gen, (1, 8, T, 128), workloads.K_OUTLIERS_4, 0.5, dtype=torch.float32)
    v = workloads.torch_kv(gen, (1, 8, T, 128), (), 0.5, dtype=torch.float32)
    q = torch.randn((1, 32, 1, 128), generator=gen, device="cuda") / np.sqrt(128)
    kk, vv, qq = (np_f32(x.to(getattr(torch, dtype))) for x in (k, v, q))
    data = make_case(kk, vv, qq, 511, dtype)
    fused = np_f32(K.pipeline("GQA_FUSED", data)).reshape(32, 128)
    tile = np_f32(K.pipeline("TILE_SDPA", data)).reshape(32, 128)
    sdpa = np_f32(K.pipeline("TORCH_SDPA", data)).reshape(32, 128)
    want, _ = oracle_out(kk, vv, qq, 511, dtype)
    for got in (fused, tile, sdpa):
        ok, err = O.within_tolerance(got, want[0], *O.TOLERANCE[dtype])
        assert ok, err


@pytest.mark.parametrize("group", [1, 2, 4, 6, 8])
def test_gqa_groups_and_int5(group):
    """Every built GQA group size, INT3, INT4 and INT5, odd block counts and tails."""
    from nsn_b200 import kernel as K
    from nsn_b200 import codec as C
    from nsn_b200 import primitives as P
    rng = np.random.default_rng(100 + group)
    from nsn_b200 import workloads
    h = 2
    for bits, nb, t in ((3, 5, 17), (5, 9, 1), (3, 1, 0), (5, 0, 40), (4, 7, 33)):
        total = nb * 64 + t
        k = workloads.np_kv(rng, (1, h, total, 128), workloads.K_OUTLIERS_8, 0.5).astype(np.float32)
        v = workloads.np_kv(rng, (1, h, total, 128), (), 1.0).astype(np.float32)
        q = rng.standard_normal((1, h * group, 1, 128)).astype(np.float16).astype(np.float32)
        kt = torch.from_numpy(k).half().cuda()
        vt = torch.from_numpy(v).half().cuda()
        qq = torch.from_numpy(q).half().cuda()
        if nb:
            g = C.encode_group(kt[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=bits)
            vg = C.encode_group(vt[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=bits)
        else:
            g = vg = None
        out = K.pipeline("GQA_FUSED", (g, kt[:, :, nb * 64:].contiguous(), qq, vg, vt[:, :, nb * 64:].contiguous()))
        want, _ = oracle_out(k, v, q, nb, "float16", bits)
        ok, err = O.within_tolerance(np_f32(out).reshape(-1, 128), want[0], *O.TOLERANCE["float16"])
        assert ok, (group, bits, nb, t, err)


def test_rejections_and_stages():
    from nsn_b200 import kernel as K
    from nsn_b200 import primitives as P
    k, v, q, nb, dt = golden_inputs("gqa4_tail")
    base = make_case(k, v, q, nb, dt)

    def mutated(fn):
        g, kt, qq, vg, vt = base
        g = dict(codes=g["codes"].clone(), metas=tuple(m.clone() for m in g["metas"]), headers=g["headers"].clone())
        vg = dict(codes=vg["codes"].clone(), metas=tuple(m.clone() for m in vg["metas"]), headers=vg["headers"].clone())
        data = [g, kt.clone(), qq.clone(), vg, vt.clone()]
        fn(data)
        return tuple(data)

    nan = float("nan")
    cases = {
        "q_nan": lambda d: d[2].view(-1)[0].fill_(nan),
        "k_tail_inf": lambda d: d[1].view(-1)[5].fill_(float("inf")),
        "v_tail_nan": lambda d: d[4].view(-1)[-1].fill_(nan),
        "k_norm_nan": lambda d: d[0]["metas"][0].view(-1)[0].fill_(nan),
        "k_min_nan": lambda d: d[0]["metas"][1].view(-1)[3].fill_(nan),
        "v_scale_inf": lambda d: d[3]["metas"][2].view(-1)[7].fill_(float("inf")),
        "v_norm_nan": lambda d: d[3]["metas"][0].view(-1)[-1].fill_(nan),
    }
    for name, fn in cases.items():
        with pytest.raises(P.NumericalFailure):
            K.pipeline("V_FUSED", mutated(fn))
        assert K.LAST_STAGE == "input_finite", name
    g, kt, qq, vg, vt = base
    with pytest.raises(P.ContractError):
        K.pipeline("V_FUSED", (g, kt, qq.float(), vg, vt))
    assert K.LAST_STAGE == "structural"
    with pytest.raises(P.ContractError):
        K.pipeline("V_FUSED", (g, kt, qq[..., :127].contiguous(), vg, vt))
    with pytest.raises(P.ContractError):
        K.pipeline("V_FUSED", (g, kt, qq, vg, torch.cat([vt, vt], 2)))
    with pytest.raises(P.ContractError):
        K.pipeline("V_FUSED", (None, kt[:, :, :0].contiguous(), qq, None, vt[:, :, :0].contiguous()))
    with pytest.raises(P.ContractError):
        K.pipeline("V_FUSED", (g, kt, qq, vg, vt.transpose(-1, -2).contiguous().transpose(-1, -2)))
    with pytest.raises(P.IntegrityError):
        K.pipeline("NOPE", base)
    # score overflow: finite inputs, non-finite scores
    big = torch.full((1, 2, 17, 128), 2.0 ** 120, dtype=torch.bfloat16, device="cuda")
    qb = torch.full((1, 8, 1, 128), 2.0 ** 120, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(P.NumericalFailure):
        K.pipeline("V_FUSED", (None, big, qb, None, big.clone()))


def test_zero_and_constant_blocks():
    """Zero norms give zero K/V rows; constant channels (scale 0) decode exactly."""
    from nsn_b200 import kernel as K
    h, nb, t = 2, 3, 5
    k = np.zeros((1, h, nb * 64 + t, 128), np.float32)
    v = np.zeros_like(k)
    k[:, :, ::2] = np.linspace(-1, 1, 128, dtype=np.float32)
    v[:, :, 1::3] = 0.5
    q = np.ones((1, h * 4, 1, 128), np.float32)
    data = make_case(k, v, q, nb, "float16")
    out = np_f32(K.pipeline("V_FUSED", data)).reshape(-1, 128)
    want, _ = oracle_out(k, v, q, nb, "float16")
    ok, err = O.within_tolerance(out, want[0])
    assert ok, err
