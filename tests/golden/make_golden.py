"""Generate the golden vectors under tests/golden/ by running the reference's own code.

Run in a container where the reference project is mounted (default
``/root/reference``; override with ``NSN_REFERENCE``):

    python tests/golden/make_golden.py

It imports the reference's torch/NumPy implementation of the path
(``experiments/nb06/source/loop_kv_nb06_primitives.py``,
``loop_kv_nb06_codec.py``, ``loop_kv_nb06_packed.py``,
``loop_kv_nb06_kernel.py`` for ``repeat_kv``, and
``papers/nsn-integrated/code/nsn_int3_core.py``), runs it on the CPU with
torch 2.11, and records inputs and outputs in ``golden.npz`` plus a JSON
index.  Nothing under tests/ reads the reference at test time; the GPU box
only sees these files.
"""
from __future__ import annotations

import base64
import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
REF = Path(os.environ.get("NSN_REFERENCE", "/root/reference"))
sys.path.insert(0, str(REF / "experiments/nb06/source"))
sys.path.insert(0, str(REF / "papers/nsn-integrated/code"))
sys.path.insert(0, str(REPO))

import loop_kv_nb06_primitives as w  # noqa: E402
w.initialize(torch, np)
import loop_kv_nb06_codec as codec  # noqa: E402
import loop_kv_nb06_packed as packed  # noqa: E402
from nsn_int3_core import nsn_int3_qdq  # noqa: E402

from nsn_b200 import workloads  # noqa: E402

PILOT_SEED = 2026093001          # experiments/ac08/source/loop_kv_pilot.py:36
torch.set_num_threads(1)

arrays: dict[str, np.ndarray] = {}
index: dict[str, dict] = {}


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


HASHED: dict[str, dict] = {}
MAX_STORED = 300_000  # bytes; larger outputs are pinned by sha256 of their raw bytes


def put(name, a, force=False, hash_only=False):
    """Store a small array verbatim; pin a large one (or a bit-exact-only output) by sha256."""
    a = np.ascontiguousarray(a)
    if (a.nbytes <= MAX_STORED or force) and not hash_only:
        arrays[name] = a
    else:
        HASHED[name] = dict(shape=list(a.shape), dtype=str(a.dtype), sha256=sha(a.tobytes()))
    return name


def tensor_bits(t: torch.Tensor) -> np.ndarray:
    """Raw bit pattern of a CPU tensor (fp16/bf16 -> uint16, fp32 -> uint32)."""
    t = t.contiguous()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy().view(np.uint32)
    return t.numpy()


# ------------------------------------------------------------------ packing KATs
def gen_pack():
    cases = []
    for bits in (3, 4, 5):
        for count in (1, 7, 63, 64, 65, 127, 128, 129, 8192):
            codes = np.random.default_rng(PILOT_SEED + count + bits).integers(0, 1 << bits, count, dtype=np.uint8)
            payload = np.frombuffer(w.pack_codes(codes, bits), np.uint8)
            back = w.unpack_codes_reference(payload, count, bits)
            assert np.array_equal(back, codes)
            key = f"pack_b{bits}_n{count}"
            put(key + "_codes", codes)
            put(key + "_bytes", payload)
            cases.append(dict(bits=bits, count=count, key=key))
    index["pack_codes"] = dict(source="loop_kv_pilot.py:370-375 codes; loop_kv_nb06_primitives.py:15-35", cases=cases)

    cases = []
    for n in (1, 2, 3, 7, 8, 9, 63, 64, 65, 8192):
        a = ((np.arange(n) * 5 + 3) % 8).astype(np.uint8)
        p = codec.pack3(torch.from_numpy(a)).numpy()
        assert p.tobytes() == w.pack_codes(a, 3)
        assert torch.equal(codec.unpack3(torch.from_numpy(p), (n,)), torch.from_numpy(a))
        put(f"pack3_n{n}_bytes", p)
        cases.append(dict(n=n, key=f"pack3_n{n}_bytes"))
    index["pack3"] = dict(source="loop_kv_pk01_cache.py:175-180 (codes (arange*5+3)%8)", cases=cases)

    a = np.repeat(np.arange(256, dtype=np.uint8), 256)
    b = np.tile(np.arange(256, dtype=np.uint8), 256)
    payload = np.stack((a, b, a ^ b), -1).reshape(-1)
    n = 65536 * 8
    gold = codec.unpack3(torch.from_numpy(payload.copy()), (n,)).numpy()
    index["byte_pairs"] = dict(source="loop_kv_pu01_kernel.py:77-80", count=n, codes_sha256=sha(gold.tobytes()))

    index["planned_bytes"] = dict(
        source="loop_kv_pilot.py:405; loop_kv_nb06_primitives.py:72-81",
        cases=[dict(shape=[1, 1, 64, 128], compressed=64, bits=4, want=w.planned_bytes((1, 1, 64, 128), 64, 4)),
               dict(shape=[1, 8, 32768, 128], compressed=511 * 64, bits=3, want=w.planned_bytes((1, 8, 32768, 128), 511 * 64, 3)),
               dict(shape=[1, 8, 1024, 128], compressed=1024, bits=3, want=w.planned_bytes((1, 8, 1024, 128), 1024, 3)),
               dict(shape=[1, 8, 131072, 128], compressed=2047 * 64, bits=5, want=w.planned_bytes((1, 8, 131072, 128), 2047 * 64, 5)),
               dict(shape=[2, 3, 200, 128], compressed=128, bits=None, want=w.planned_bytes((2, 3, 200, 128), 128, None))])


# ------------------------------------------------------------------ encode / decode
def encode_case(name, x: torch.Tensor, bits_list=(3, 4, 5), note=""):
    """Record nsn_encode/nsn_decode of the reference on x (any layout)."""
    entry = dict(shape=list(x.shape), dtype=str(x.dtype).replace("torch.", ""),
                 contiguous=bool(x.is_contiguous()), channel_stride=int(x.stride(-1)), note=note, bits={})
    put(f"enc_{name}_x", tensor_bits(x))
    for bits in bits_list:
        rec = {}
        try:
            q, metas = w.nsn_encode(x, bits)
        except w.NumericalFailure as e:
            rec["raises"] = "NumericalFailure"
            rec["message"] = str(e)
            entry["bits"][str(bits)] = rec
            continue
        key = f"enc_{name}_b{bits}"
        put(key + "_packed", np.frombuffer(w.pack_codes(q.numpy(), bits), np.uint8))
        for tag, m in zip(("n", "m", "s"), metas):
            put(key + "_" + tag, tensor_bits(m))
        for dt in (torch.float16, torch.bfloat16, torch.float32):
            tag = str(dt).replace("torch.", "")
            try:
                y = w.nsn_decode(q, metas, dt)
                put(f"{key}_dec_{tag}", tensor_bits(y), hash_only=True)
                rec["dec_" + tag] = True
            except w.NumericalFailure as e:
                rec["dec_" + tag] = "NumericalFailure: " + str(e)
        if bits == 3:
            y = nsn_int3_qdq(x)
            put(f"{key}_int3_qdq", tensor_bits(y), hash_only=True)
            rec["int3_qdq_equals_nsn_qdq"] = bool(torch.equal(y, w.nsn_qdq(x, 3)))
        rec["key"] = key
        entry["bits"][str(bits)] = rec
    index.setdefault("encode", {})[name] = entry


def gen_encode():
    fix = json.loads((REF / "scripts/nb06_codec_fixture.json").read_text())
    for bname, blk in fix["blocks"].items():
        raw = base64.b64decode(blk["data_base64"], validate=True)
        assert sha(raw) == blk["sha256"]
        a = np.frombuffer(raw, dtype="<u2").copy().reshape(blk["shape"])
        x = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).reshape(1, 8, 1, 64, 128)
        encode_case("fixture_" + bname, x, note="scripts/nb06_codec_fixture.json real Nanbeige block")

    gen = torch.Generator(device="cpu").manual_seed(PILOT_SEED)
    encode_case("zeros", torch.zeros(1, 2, 1, 64, 128))
    encode_case("ones", torch.ones(1, 2, 1, 64, 128))
    encode_case("strided", torch.randn(1, 2, 1, 128, 64, generator=gen).transpose(-1, -2), note="channel axis strided")
    encode_case("strided_bf16", torch.randn(1, 2, 1, 128, 64, generator=gen).transpose(-1, -2).to(torch.bfloat16))
    encode_case("two_blocks_fp32", torch.randn(2, 64, 128, generator=gen))

    k, v, _, _, _ = workloads.np_config(0)
    kt = torch.from_numpy(k).reshape(1, 8, 16, 64, 128)
    vt = torch.from_numpy(v).reshape(1, 8, 16, 64, 128)
    index["cfg0_inputs"] = dict(k_sha256=sha(k.tobytes()), v_sha256=sha(v.tobytes()), shape=list(k.shape))
    encode_case("cfg0_k", kt, note="cfg0 K fp16 (regenerated from workloads.np_config(0))")
    encode_case("cfg0_v", vt, note="cfg0 V fp16")

    # Edge cases: constant channels (s == 0), one nonzero token, mixed zero-norm tokens,
    # wide dynamic range, and the rejection fixtures.
    x = torch.randn(1, 1, 1, 64, 128, generator=gen)
    x[..., :, 5] = 0.25
    x[..., :, 77] = -1.0
    encode_case("const_channels", x.to(torch.float16))
    x = torch.zeros(1, 1, 1, 64, 128)
    x[..., 17, :] = torch.randn(128, generator=gen)
    encode_case("one_token", x.to(torch.float16))
    x = torch.randn(1, 1, 2, 64, 128, generator=gen) * torch.exp(torch.randn(1, 1, 2, 64, 1, generator=gen) * 3)
    x[..., ::3, :] = 0
    encode_case("zero_norm_rows", x.to(torch.float16))
    x = torch.randn(1, 1, 1, 64, 128, generator=gen) * torch.exp(torch.randn(1, 1, 1, 64, 1, generator=gen) * 4)
    encode_case("huge_range_fp32", x, note="some token norm overflows fp16 -> must raise")
    x = torch.randn(1, 1, 1, 64, 128, generator=gen) * torch.exp(torch.randn(1, 1, 1, 64, 1, generator=gen) * 1.5)
    encode_case("wide_range_fp32", x)
    encode_case("overflow_1e5", torch.full((64, 128), 1e5), note="loop_kv_pilot.py:391-396 must raise")
    x = torch.randn(1, 1, 1, 64, 128, generator=gen)
    x[..., 9, :] = 1e-9
    encode_case("norm_underflow", x, note="token norm underflows fp16 -> must raise")
    x = torch.randn(1, 1, 1, 64, 128, generator=gen)
    x[..., 3, 7] = float("nan")
    encode_case("nan_input", x, note="non-finite input must raise")

    # Round-trip ties: values on exact rounding boundaries.
    x = torch.linspace(-1, 1, 64 * 128).reshape(1, 1, 1, 64, 128)
    encode_case("linspace", x)

    # Channels whose smallest value is a zero of either sign (the min meta's sign is
    # decided by the reduction's tie rule); the last 16 channels also hold negatives.
    g2 = torch.Generator().manual_seed(PILOT_SEED + 11)
    x = torch.rand(1, 1, 2, 64, 128, generator=g2) + 0.1
    zero = torch.rand(1, 1, 2, 64, 128, generator=g2) < 0.1
    neg = torch.rand(1, 1, 2, 64, 128, generator=g2) < 0.5
    x = torch.where(zero, torch.where(neg, torch.tensor(-0.0), torch.tensor(0.0)), x)
    x[..., 112:] -= 0.6
    encode_case("signed_zero_min", x.to(torch.float16))
    encode_case("signed_zero_min_bf16", x.to(torch.bfloat16))


# ------------------------------------------------------------------ encode_group / restore_group
def gen_group():
    k, v, q, _, _ = workloads.np_config(0)
    out = {}
    for name, src in (("cfg0_k", k), ("cfg0_v", v)):
        x = torch.from_numpy(src).reshape(1, 8, 16, 64, 128)
        g = codec.encode_group(x, 0)
        put(f"group_{name}_codes", g["codes"].numpy())
        put(f"group_{name}_headers", g["headers"].numpy())
        for tag, m in zip(("n", "m", "s"), g["metas"]):
            put(f"group_{name}_{tag}", tensor_bits(m))
        for dt in (torch.float16, torch.bfloat16):
            y = codec.restore_group(g, dt)
            put(f"group_{name}_restore_{str(dt).replace('torch.', '')}", tensor_bits(y), hash_only=True)
        g2 = codec.encode_group(x[:, :, :5], 320)
        put(f"group_{name}_headers_start320", g2["headers"].numpy())
        out[name] = dict(codes_shape=list(g["codes"].shape))
    index["group"] = out


# ------------------------------------------------------------------ bridge attention
def bridge(q16, kfull, vfull):
    """Reference bridge: repeat_kv + SDPA on the CPU (loop_kv_nb06_kernel.py:156-174)."""
    import loop_kv_nb06_kernel as kern
    rep = q16.shape[1] // kfull.shape[1]
    kk = kern.repeat_kv(kfull, rep)
    vv = kern.repeat_kv(vfull, rep)
    out = torch.nn.functional.scaled_dot_product_attention(q16, kk, vv, attn_mask=None, dropout_p=0.0, is_causal=False)
    # finish(): explicit fp32 softmax.V (loop_kv_ac08_attention.py:38-44 style)
    s = torch.matmul(q16.float(), kk.float().transpose(-2, -1)) * (128 ** -0.5)
    p = torch.softmax(s, -1)
    fin = torch.matmul(p, vv.float())
    return out.transpose(1, 2).contiguous(), fin.transpose(1, 2).contiguous()


def attn_case(name, k, v, q, nb, t, dtype=torch.float16):
    """k,v [1,H,T,128] fp16 numpy; the first nb*64 tokens are sealed with INT3."""
    h = k.shape[1]
    kt = torch.from_numpy(k).to(dtype)
    vt = torch.from_numpy(v).to(dtype)
    qt = torch.from_numpy(q).to(dtype)
    fulls = []
    for tag, src in (("k", kt), ("v", vt)):
        put(f"attn_{name}_{tag}_in", tensor_bits(src))
        if nb:
            g = codec.encode_group(src[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0)
            rest = codec.restore_group(g, dtype)
            full = torch.cat((rest, src[:, :, nb * 64:]), 2)
        else:
            full = src
        fulls.append(full)
    out, fin = bridge(qt, fulls[0], fulls[1])
    put(f"attn_{name}_q", tensor_bits(qt))
    put(f"attn_{name}_sdpa", tensor_bits(out))
    put(f"attn_{name}_finish", tensor_bits(fin))
    index.setdefault("attention", {})[name] = dict(h=h, hq=q.shape[1], blocks=nb, tail=t, dtype=str(dtype).replace("torch.", ""))


def gen_attention():
    k, v, q, nb, t = workloads.np_config(0)
    attn_case("cfg0", k, v, q, nb, t)
    rng = np.random.default_rng(11)
    for name, h, hq, nb, t, dt in (("mha_tail", 2, 2, 3, 37, torch.float16),
                                   ("gqa4_tail", 2, 8, 2, 64, torch.float16),
                                   ("gqa8_bf16", 1, 8, 4, 5, torch.bfloat16),
                                   ("tail_only", 2, 8, 0, 17, torch.float16),
                                   ("gqa6", 2, 12, 2, 1, torch.bfloat16)):
        total = nb * 64 + t
        kk = workloads.np_kv(rng, (1, h, total, 128), workloads.K_OUTLIERS_4, 0.5)
        vv = workloads.np_kv(rng, (1, h, total, 128), (), 0.5)
        qq = rng.standard_normal((1, hq, 1, 128), dtype=np.float32).astype(np.float16)
        attn_case(name, kk, vv, qq, nb, t, dt)


# ------------------------------------------------------------------ packed cache lifecycle
class FixtureBase:
    """Minimal stand-in for the HF DynamicCache surface PackedCache uses."""

    def __init__(self):
        self.key_cache = []
        self.value_cache = []
        self._seen_tokens = 0

    def get_seq_length(self, layer_idx=0):
        return 0 if layer_idx >= len(self.key_cache) or self.key_cache[layer_idx] is None else self.key_cache[layer_idx].shape[-2]

    def update(self, k, v, i, cache_kwargs=None):
        while len(self.key_cache) <= i:
            self.key_cache.append(None)
            self.value_cache.append(None)
        for data, x in ((self.key_cache, k), (self.value_cache, v)):
            data[i] = x if data[i] is None else torch.cat((data[i], x), -2)
        return self.key_cache[i], self.value_cache[i]


def gen_cache():
    old = (w.LAYERS, w.HEADS)
    try:
        w.LAYERS, w.HEADS = 2, 2
        r = 1
        cache = packed.make_packed_cache(FixtureBase)(r, 3)
        gen = torch.Generator(device="cpu").manual_seed(PILOT_SEED + 7)
        slots = w.LAYERS * r
        x = torch.randn(slots, 2, 300, 128, generator=gen).to(torch.bfloat16)
        put("cache_x", tensor_bits(x))
        prefill = 200
        trace = []
        returned = {}
        for end in [prefill] + list(range(prefill + 1, 300 + 1)):
            start = 0 if end == prefill else end - 1
            for s in range(slots):
                k = x[s:s + 1, :, start:end, :]
                v = (k.float() * .75).to(torch.bfloat16)
                pos = {"cache_position": torch.arange(start, end)}
                rk, rv = cache.update(k, v, s, pos)
                if end in (prefill, 201, 263, 264, 265, 300):
                    returned[(end, s)] = (rk, rv)
            if end == prefill:
                cache.post_prefill()
            else:
                cache.post_decode()
            trace.append(dict(end=end, compressed=cache.compressed.get(0, 0), tail=cache.key_cache[0].shape[-2]))
        for (end, s), (rk, rv) in returned.items():
            put(f"cache_ret_{end}_{s}_k", tensor_bits(rk), hash_only=True)
            put(f"cache_ret_{end}_{s}_v", tensor_bits(rv), hash_only=True)
        for s in range(slots):
            for kv in ("K", "V"):
                g = cache.packed[(s, kv)]
                put(f"cache_final_{s}_{kv}_codes", g["codes"].numpy())
                put(f"cache_final_{s}_{kv}_headers", g["headers"].numpy())
                for tag, m in zip(("n", "m", "s"), g["metas"]):
                    put(f"cache_final_{s}_{kv}_{tag}", tensor_bits(m))
                tail = (cache.key_cache if kv == "K" else cache.value_cache)[s]
                put(f"cache_final_{s}_{kv}_tail", tensor_bits(tail))
        index["cache"] = dict(source="loop_kv_nb06_packed.py:5-61 with LAYERS,HEADS=2,2, r=1", slots=slots,
                              prefill=prefill, last=300, checkpoints=[200, 201, 263, 264, 265, 300],
                              trace=trace, final_compressed=cache.compressed.get(0, 0))
    finally:
        w.LAYERS, w.HEADS = old


# ------------------------------------------------------------------ library INT3 container (src/nsn)
def gen_int3asym():
    sys.path.insert(0, str(REF / "src"))
    from nsn.cache import Int3AsymNsepPchanCache
    from nsn.pack import pack_int3_unsigned
    g2 = torch.Generator().manual_seed(PILOT_SEED + 21)
    cases = []

    def case(name, x):
        c = Int3AsymNsepPchanCache.from_fp16(x)
        y = c.to_fp16()
        put(f"asym_{name}_x", tensor_bits(x))
        put(f"asym_{name}_packed", c.packed_d.numpy())
        put(f"asym_{name}_norm", tensor_bits(c.norm))
        put(f"asym_{name}_dmin", tensor_bits(c.d_min))
        put(f"asym_{name}_dstep", tensor_bits(c.d_step))
        put(f"asym_{name}_y", tensor_bits(y))
        cases.append(dict(name=name, shape=list(x.shape), dtype=str(x.dtype).replace("torch.", ""),
                          channel_stride=int(x.stride(-1)), size_bytes=int(c.size_bytes())))

    x = torch.randn(1, 2, 70, 128, generator=g2) * torch.exp(torch.randn(1, 2, 70, 1, generator=g2))
    x[..., 5] *= 8
    case("fp16_128", x.half())
    case("fp32_64", torch.randn(2, 1, 33, 64, generator=g2))
    case("fp16_256", (torch.randn(1, 1, 130, 256, generator=g2) * 3).half())
    case("bf16_128", torch.randn(1, 1, 65, 128, generator=g2).to(torch.bfloat16))
    case("fp16_128_strided", torch.randn(1, 2, 128, 40, generator=g2).half().transpose(-1, -2))
    x = torch.randn(1, 1, 48, 128, generator=g2)
    x[..., ::7, :] = 0
    x[..., 3] = 0.5
    case("zero_tokens_const_channel", x.half())
    x = torch.rand(1, 1, 64, 128, generator=g2) + 0.1
    zero = torch.rand(1, 1, 64, 128, generator=g2) < 0.1
    neg = torch.rand(1, 1, 64, 128, generator=g2) < 0.5
    x = torch.where(zero, torch.where(neg, torch.tensor(-0.0), torch.tensor(0.0)), x)
    case("signed_zero_min", x.half())
    codes = torch.randint(0, 8, (3, 5, 64), generator=g2, dtype=torch.int8)
    put("asym_pack_codes", codes.numpy())
    put("asym_pack_bytes", pack_int3_unsigned(codes).numpy())
    index["int3asym"] = dict(source="src/nsn/cache.py:134-313; src/nsn/pack.py:85-163", cases=cases)


# ------------------------------------------------------------------ K1c batched decode scores
def gen_k1c():
    sys.path.insert(0, str(REF / "experiments/kernels"))
    import phase_k1c_triton_fused_kernel as k1c
    models = {"gemma": k1c.GRID_MODELS[0], "qwen": k1c.GRID_MODELS[1]}
    cells = []
    for mname, model in models.items():
        for recipe, bits in (("nsn", 5), ("kivi", 5), ("nsn", 4), ("kivi", 4), ("fp16", 16)):
            B, T = 2, 97
            q, ref_store, tstore, n_q, n_kv, hd = k1c.make_triton_store(model, B, T, bits, recipe, "cpu")
            ref32 = k1c._torch_decode_scores(q.float(), {k: (v.float() if torch.is_tensor(v) else v)
                                                        for k, v in ref_store.items()}, recipe, n_q, n_kv, hd)
            key = f"k1c_{mname}_{recipe}{bits}"
            arrays_sha = {}
            for f in ("code", "min", "step", "eff_norm"):
                if f in tstore:
                    arrays_sha[f] = sha(tensor_bits(tstore[f]).tobytes())
            put(key + "_scores", ref32.numpy(), force=True)
            cells.append(dict(key=key, model=mname, recipe=recipe, bits=bits, B=B, T=T, q_sha256=sha(tensor_bits(q).tobytes()),
                              store_sha256=arrays_sha))
    index["k1c"] = dict(source="experiments/kernels/phase_k1c_triton_fused_kernel.py:63-250", gate_tol=k1c.GATE_TOL,
                        cells=cells)


def main():
    gen_pack()
    gen_encode()
    gen_group()
    gen_attention()
    gen_cache()
    gen_int3asym()
    gen_k1c()
    np.savez_compressed(HERE / "golden.npz", **arrays)
    index["hashed"] = HASHED
    index["torch"] = torch.__version__
    index["cpu_capability"] = torch.backends.cpu.get_cpu_capability()
    index["npz_sha256"] = sha((HERE / "golden.npz").read_bytes())
    (HERE / "golden.json").write_text(json.dumps(index, indent=1, sort_keys=True) + "\n")
    print("wrote", len(arrays), "arrays;", (HERE / "golden.npz").stat().st_size, "bytes")


if __name__ == "__main__":
    main()
