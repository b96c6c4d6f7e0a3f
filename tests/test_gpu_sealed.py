"""GPU parity of the paged cache's default attention path (restore_rounding="k"):
sealed INT3 blocks on attn_sealed_kernel (K rows restored and rounded to the cache dtype
as the reference bridge rounds them, V the exact fp32 restore), tails on
attn_native_rows_kernel, then attn_merge_kernel.

The contract is the reference bridge, restore_group(g, dtype) + SDPA
(experiments/nb06/source/loop_kv_nb06_codec.py:36-38, loop_kv_nb06_kernel.py:156-174),
at the parity bar of oracle.TOLERANCE.  Checked here:
* every golden attention case recorded from the reference (tests/golden), through the
  cache, against the reference's own SDPA output;
* GQA groups 1..8, fp16 and bf16 caches, queries scaled by 1/sqrt(128) and unscaled,
  against fp64 attention over the bridge's rows (K and V rounded);
* the fp32 context against fp64 attention over K rounded and V exact, the arithmetic the
  kernel implements, with a bar a little above fp32 accumulation;
* the full-size cfg1 sequence (511 blocks + 64 tail tokens) and the full cfg2 benchmark
  state (64 sequences, 32-block chunks, 64 decode steps through PagedKVCache.step, the
  native step plan, with a seal per step on average), against the fp64 oracle on a sample
  of sequences and steps; the cfg2 state also through
  restore_rounding="exact" (the benchmark's headline kernel), whose parity with the bridge
  holds for the benchmark's 1/sqrt(128)-scaled queries.
"""
import numpy as np
import pytest
import torch

import golden_util as G
from oracle import nsn_oracle as O

pytestmark = pytest.mark.gpu

# fp32 context against fp64 attention over (K rounded, V exact): fp32 accumulation plus the
# rare restored K value that lands on the other side of a rounding tie of the cache dtype
# (the kernel forms alpha * d, the bridge n * (d / ||d||): the same value up to two fp32
# roundings)
KROUND = (2e-4, 5e-5)
DT = {"float16": torch.float16, "bfloat16": torch.bfloat16}


class Restored:
    """The oracle's restores of a sequence's blocks, encoded once: rows(T, nb, kind) is
    K or V [h, T, 128] in fp64 with the first nb blocks restored as `kind` ("bridge":
    rounded to dtype like restore_group; "exact": the fp32 restore before the cast) and
    the rest of the T tokens native."""

    def __init__(self, src, nb_max, dtype, bits=3):
        self.src, self.dtype = src, dtype
        h = src.shape[0]
        self.y = {}
        if nb_max:
            x = src[None, :, :nb_max * 64].astype(np.float32).reshape(1, h, nb_max, 64, 128)
            q8, n, m, s, st = O.nsn_encode(x, bits)
            assert st == 0
            self.y["bridge"] = np.asarray(O.nsn_decode(q8, n, m, s, dtype), np.float32).reshape(h, nb_max * 64, 128)
            self.y["exact"] = np.asarray(O.nsn_decode(q8, n, m, s, np.float32), np.float32).reshape(h, nb_max * 64, 128)

    def rows(self, T, nb, kind):
        parts = [self.y[kind][:, :nb * 64]] if nb else []
        parts.append(self.src[:, nb * 64:T])
        return np.concatenate(parts, 1).astype(np.float64)


def rows(src, nb, dtype, kind, bits=3):
    return Restored(src, nb, dtype, bits).rows(src.shape[1], nb, kind)


def attention64(q, k, v):
    """q [hq,128], k/v [h,T,128] fp64 -> [hq,128] (repeat_kv grouping, scale 1/sqrt(128))."""
    rep = q.shape[0] // k.shape[0]
    out = np.empty((q.shape[0], 128))
    for j in range(q.shape[0]):
        s = k[j // rep] @ q[j] / np.sqrt(128.0)
        p = np.exp(s - s.max())
        out[j] = (p[:, None] * v[j // rep]).sum(0) / p.sum()
    return out


def vexact_bar(q, k, v):
    """The V codes enter mma.sync as fp16 subnormals; allow 2^-16 of the largest |v|."""
    return 2.0 ** -16 * np.abs(v).max()


def fill(cache, b, k, v, tail64=False):
    """Load sequence b from K/V [h, T, 128] (float32 values of the cache dtype).

    With tail64 the last 64 tokens stay native: the cache keeps at most 63 between steps,
    so T - 1 tokens are prefilled and the last one is returned as the (k_new, v_new)
    [1, h, 128] pair for attend to append; otherwise returns (None, None)."""
    dt = cache.dtype
    if tail64:
        assert k.shape[1] % 64 == 0 and k.shape[1] > 0
        cache.prefill(b, torch.from_numpy(k[:, :-1]).cuda().to(dt), torch.from_numpy(v[:, :-1]).cuda().to(dt))
        return (torch.from_numpy(k[:, -1].copy()).cuda().to(dt)[None],
                torch.from_numpy(v[:, -1].copy()).cuda().to(dt)[None])
    cache.prefill(b, torch.from_numpy(k).cuda().to(dt), torch.from_numpy(v).cuda().to(dt))
    return None, None


def new_cache(batch, h, hq, max_blocks, dtype, mode="k", bits=3):
    from nsn_b200.paged import PagedKVCache
    return PagedKVCache(batch, h, max_blocks=max_blocks, bits=bits, dtype=dtype, hq=hq, restore_rounding=mode)


def exact_k_bar(q, k, v):
    """The exact kernel (restore_rounding="exact") takes the K codes as fp16-subnormal MMA
    operands as well; its logits carry up to ~2^-16 * sum_c |q_c k_c| / sqrt(128), which
    moves an output by at most that times max |v|."""
    rep = q.shape[0] // k.shape[0]
    sabs = np.einsum("jd,jtd->jt", np.abs(q), np.abs(np.repeat(k, rep, 0))).max() / np.sqrt(128.0)
    return 2.0 ** -16 * sabs * np.abs(v).max()


@pytest.mark.parametrize("name", sorted(G.index()["attention"]))
def test_golden_attention_through_default_cache(name):
    """The reference's recorded SDPA output of every golden case, through PagedKVCache."""
    e = G.index()["attention"][name]
    dt = e["dtype"]
    h, hq, nb, t = e["h"], e["hq"], e["blocks"], e["tail"]
    if name == "cfg0":
        from nsn_b200 import workloads
        k, v, q, _, _ = workloads.np_config(0)
        k, v, q = k[0].astype(np.float32), v[0].astype(np.float32), q.astype(np.float32)
        assert G.matches("attn_cfg0_q", q.astype(np.float16).view(np.uint16))
    else:
        k = G.bits_to_float32(G.get(f"attn_{name}_k_in"), dt).reshape(h, -1, 128)
        v = G.bits_to_float32(G.get(f"attn_{name}_v_in"), dt).reshape(h, -1, 128)
        q = G.bits_to_float32(G.get(f"attn_{name}_q"), dt)
    q = q.reshape(1, hq, 128)
    assert k.shape[1] == nb * 64 + t
    # a 64-token native tail stays native: 63 prefilled + 1 appended (not sealed)
    cache = new_cache(1, h, hq, nb + 1, DT[dt])
    extra = fill(cache, 0, k, v, tail64=(t == 64))
    assert int(cache.n_blocks[0]) == nb
    assert cache.uses_alpha_path()
    out = cache.attend(torch.from_numpy(q).cuda().to(DT[dt]), *extra)
    cache.check()
    want = G.bits_to_float32(G.get(f"attn_{name}_sdpa"), dt).reshape(1, hq, 128)
    ok, err = O.within_tolerance(out.float().cpu().numpy(), want, *O.TOLERANCE[dt])
    assert ok, (name, err)


@pytest.mark.parametrize("h,hq,dtype", [(2, 8, "float16"), (2, 6, "float16"), (1, 8, "float16"), (3, 3, "float16"),
                                        (2, 12, "float16"), (2, 16, "bfloat16"), (2, 8, "bfloat16"),
                                        (4, 4, "bfloat16")])
@pytest.mark.parametrize("q_scale", [1.0, float(np.sqrt(128))])
def test_default_path_matches_bridge(h, hq, dtype, q_scale):
    from nsn_b200 import workloads
    rng = np.random.default_rng(hq * 31 + h + (7 if dtype == "bfloat16" else 0) + int(q_scale))
    lens = [64, 1, 130, 64 * 9 + 17, 64 * 21, 64 * 5 + 63, 64 * 33 + 40]
    cache = new_cache(len(lens), h, hq, 34, DT[dtype])
    assert cache.uses_alpha_path()
    hk, hv = [], []
    for b, L in enumerate(lens):
        k = workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32)
        v = workloads.np_kv(rng, (h, L, 128), (), 0.5).astype(np.float32)
        if dtype == "bfloat16":  # values of the cache dtype
            k, v = O.cast(k, "bfloat16"), O.cast(v, "bfloat16")
        hk.append(k)
        hv.append(v)
        fill(cache, b, k, v)
    q = (rng.standard_normal((len(lens), hq, 128)) * q_scale / np.sqrt(128)).astype(np.float32)
    q = O.cast(q, dtype).astype(np.float32)
    out32 = torch.empty((len(lens), hq, 128), dtype=torch.float32, device="cuda")
    out = cache.attend(torch.from_numpy(q).cuda().to(DT[dtype]), out_f32=out32)
    cache.check()
    got, got32 = out.float().cpu().numpy(), out32.cpu().numpy()
    for b, L in enumerate(lens):
        nb = L // 64
        q64 = q[b].astype(np.float64)
        kb, vb = rows(hk[b], nb, dtype, "bridge"), rows(hv[b], nb, dtype, "bridge")
        ok, err = O.within_tolerance(got[b], attention64(q64, kb, vb), *O.TOLERANCE[dtype])
        assert ok, ("bridge", b, L, err)
        vx = rows(hv[b], nb, dtype, "exact")
        ok, err = O.within_tolerance(got32[b], attention64(q64, kb, vx), KROUND[0], KROUND[1] + vexact_bar(q64, kb, vx))
        assert ok, ("k rounded, v exact", b, L, err)


@pytest.mark.parametrize("h,hq,dtype", [(8, 64, "float16"), (2, 16, "float16"), (2, 12, "bfloat16"),
                                        (2, 8, "float16"), (1, 1, "bfloat16")])
@pytest.mark.parametrize("q_scale", [1.0, float(np.sqrt(128))])
def test_int5_default_path_matches_bridge(h, hq, dtype, q_scale):
    """INT5 caches on the tensor-core kernel: the same contract and the same data as the INT3
    cases above (K rounded like the bridge, V exact), through the INT5 code windows (codes at
    window bits 6 and 7 shifted down).  The fp16 and fp32 cfg4 data (8 outlier channels,
    V sigma 1) is covered by the step and full-size tests below."""
    from nsn_b200 import workloads
    rng = np.random.default_rng(hq * 37 + h + (5 if dtype == "bfloat16" else 0) + int(q_scale))
    lens = [64, 1, 130, 64 * 9 + 17, 64 * 21, 64 * 5 + 63]
    cache = new_cache(len(lens), h, hq, 22, DT[dtype], bits=5)
    assert cache.uses_alpha_path()
    hk, hv = [], []
    for b, L in enumerate(lens):
        k = workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32)
        v = workloads.np_kv(rng, (h, L, 128), (), 0.5).astype(np.float32)
        if dtype == "bfloat16":
            k, v = O.cast(k, "bfloat16"), O.cast(v, "bfloat16")
        hk.append(k)
        hv.append(v)
        fill(cache, b, k, v)
    q = (rng.standard_normal((len(lens), hq, 128)) * q_scale / np.sqrt(128)).astype(np.float32)
    q = O.cast(q, dtype).astype(np.float32)
    out32 = torch.empty((len(lens), hq, 128), dtype=torch.float32, device="cuda")
    out = cache.attend(torch.from_numpy(q).cuda().to(DT[dtype]), out_f32=out32)
    cache.check()
    got, got32 = out.float().cpu().numpy(), out32.cpu().numpy()
    for b, L in enumerate(lens):
        nb = L // 64
        q64 = q[b].astype(np.float64)
        kb, vb = rows(hk[b], nb, dtype, "bridge", 5), rows(hv[b], nb, dtype, "bridge", 5)
        ok, err = O.within_tolerance(got[b], attention64(q64, kb, vb), *O.TOLERANCE[dtype])
        assert ok, ("bridge", b, L, err)
        vx = rows(hv[b], nb, dtype, "exact", 5)
        ok, err = O.within_tolerance(got32[b], attention64(q64, kb, vx), KROUND[0], KROUND[1] + vexact_bar(q64, kb, vx))
        assert ok, ("k rounded, v exact", b, L, err)


def test_int5_cache_steps_and_seals():
    """An INT5 paged cache stepped through nsnkv_paged_step: the seal writes INT5 records,
    and every output matches the bridge over the sequence so far."""
    from nsn_b200 import workloads
    rng = np.random.default_rng(29)
    h, hq, lens, steps = 2, 16, [100, 63, 64 * 3], 70
    cache = new_cache(len(lens), h, hq, 6, torch.float16, bits=5)
    hk = [workloads.np_kv(rng, (h, L + steps, 128), workloads.K_OUTLIERS_8, 0.5).astype(np.float32) for L in lens]
    hv = [workloads.np_kv(rng, (h, L + steps, 128), (), 1.0).astype(np.float32) for L in lens]
    for b, L in enumerate(lens):
        fill(cache, b, hk[b][:, :L], hv[b][:, :L])
    for s in range(steps):
        q = (rng.standard_normal((len(lens), hq, 128)) / np.sqrt(128)).astype(np.float16)
        kn = torch.from_numpy(np.stack([hk[b][:, lens[b] + s] for b in range(len(lens))])).cuda().half()
        vn = torch.from_numpy(np.stack([hv[b][:, lens[b] + s] for b in range(len(lens))])).cuda().half()
        out = cache.step(torch.from_numpy(q).cuda(), kn, vn).float().cpu().numpy()
        if s in (0, 1, 36, 69):
            for b, L in enumerate(lens):
                T = L + s + 1
                nb = (T - 1) // 64
                src_k, src_v = hk[b][:, :T], hv[b][:, :T]
                kb, vb = rows(src_k, nb, "float16", "bridge", 5), rows(src_v, nb, "float16", "bridge", 5)
                ok, err = O.within_tolerance(out[b], attention64(q[b].astype(np.float64), kb, vb),
                                             *O.TOLERANCE["float16"])
                assert ok, (s, b, err)
    cache.check()
    assert cache.n_blocks.cpu().tolist() == [(L + steps) // 64 for L in lens]


def test_int4_cache_steps_on_the_restore_kernel():
    """INT4 caches (no tensor-core kernel) step through the plan on the restore kernel, K and
    V rounded like the bridge, with the seal's counter kernel (no renorm factors)."""
    from nsn_b200 import workloads
    rng = np.random.default_rng(31)
    h, hq, lens, steps = 2, 8, [70, 127], 66
    cache = new_cache(len(lens), h, hq, 5, torch.float16, bits=4)
    assert not cache.uses_alpha_path()
    hk = [workloads.np_kv(rng, (h, L + steps, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32) for L in lens]
    hv = [workloads.np_kv(rng, (h, L + steps, 128), (), 0.5).astype(np.float32) for L in lens]
    for b, L in enumerate(lens):
        fill(cache, b, hk[b][:, :L], hv[b][:, :L])
    for s in range(steps):
        q = (rng.standard_normal((len(lens), hq, 128)) / np.sqrt(128)).astype(np.float16)
        kn = torch.from_numpy(np.stack([hk[b][:, lens[b] + s] for b in range(len(lens))])).cuda().half()
        vn = torch.from_numpy(np.stack([hv[b][:, lens[b] + s] for b in range(len(lens))])).cuda().half()
        out = cache.step(torch.from_numpy(q).cuda(), kn, vn).float().cpu().numpy()
        if s in (0, 57, 65):
            for b, L in enumerate(lens):
                T = L + s + 1
                nb = (T - 1) // 64
                kb = rows(hk[b][:, :T], nb, "float16", "bridge", 4)
                vb = rows(hv[b][:, :T], nb, "float16", "bridge", 4)
                ok, err = O.within_tolerance(out[b], attention64(q[b].astype(np.float64), kb, vb),
                                             *O.TOLERANCE["float16"])
                assert ok, (s, b, err)
    cache.check()
    assert cache.n_blocks.cpu().tolist() == [(L + steps) // 64 for L in lens]


def test_cfg4_full_size_split_kv():
    """cfg4 at full size (2047 INT5 blocks + 64 tail tokens, GQA 64:8) through the split-KV
    path on block records: two shards on one GPU, their (o, lse) records merged, against the
    bridge over the whole sequence."""
    from nsn_b200 import codec, workloads
    from nsn_b200.splitkv import ShardedSequence, merge_records, shard_range
    c = workloads.CONFIGS[4]
    h, hq, nb, t = c["h"], c["hq"], c["blocks"], 64
    gen = torch.Generator(device="cuda").manual_seed(41)
    T = nb * 64 + t
    k = workloads.torch_kv(gen, (1, h, T, 128), c["k_outliers"], 0.5)
    v = workloads.torch_kv(gen, (1, h, T, 128), (), c["v_sigma"])
    q = (torch.randn((1, hq, 1, 128), generator=gen, device="cuda") / np.sqrt(128)).half()
    g = codec.encode_group(k[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=5)
    vg = codec.encode_group(v[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=5)
    kt, vt = k[:, :, nb * 64:].contiguous(), v[:, :, nb * 64:].contiguous()
    world, recs = 2, []
    for r in range(world):
        s, e = shard_range(nb, world, r)
        sub = lambda gr: dict(codes=gr["codes"][:, :, s:e].contiguous(),
                              metas=tuple(m[:, :, s:e].contiguous() for m in gr["metas"]))
        last = r == world - 1
        sh = ShardedSequence(sub(g), sub(vg), kt if last else None, vt if last else None, h, hq, 5)
        assert sh.kp is not None and "alpha" in sh.kp  # the tensor-core path
        o, lse = sh.local(q)
        sh.check()
        recs.append(torch.cat([o.reshape(-1), lse.reshape(-1)]))
    out, status = merge_records(torch.cat(recs), world, hq, dtype=torch.float16)
    assert int(status.item()) == 0
    got = out.float().cpu().numpy().reshape(hq, 128)
    q64 = q.float().cpu().numpy().reshape(hq, 128).astype(np.float64)
    kk, vv = k[0].float().cpu().numpy(), v[0].float().cpu().numpy()
    kb, vb = rows(kk, nb, "float16", "bridge", 5), rows(vv, nb, "float16", "bridge", 5)
    ok, err = O.within_tolerance(got, attention64(q64, kb, vb), *O.TOLERANCE["float16"])
    assert ok, err


def test_default_path_q_magnitudes():
    """Tiny and large queries: q is the Q.K mma's B operand as it is, no exponent shift."""
    from nsn_b200 import workloads
    for q_scale in (1e-3, 300.0, 4000.0):
        rng = np.random.default_rng(5)
        lens = [64 * 12 + 5, 64 * 4]
        cache = new_cache(2, 2, 8, 13, torch.float16)
        hk = [workloads.np_kv(rng, (2, L, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32) for L in lens]
        hv = [workloads.np_kv(rng, (2, L, 128), (), 0.5).astype(np.float32) for L in lens]
        for b in range(2):
            fill(cache, b, hk[b], hv[b])
        q = (rng.standard_normal((2, 8, 128)) * q_scale / np.sqrt(128)).astype(np.float16).astype(np.float32)
        out32 = torch.empty((2, 8, 128), dtype=torch.float32, device="cuda")
        cache.attend(torch.from_numpy(q).cuda().half(), out_f32=out32)
        cache.check()
        for b, L in enumerate(lens):
            q64 = q[b].astype(np.float64)
            kb, vx = rows(hk[b], L // 64, "float16", "bridge"), rows(hv[b], L // 64, "float16", "exact")
            ok, err = O.within_tolerance(out32[b].cpu().numpy(), attention64(q64, kb, vx), KROUND[0],
                                         KROUND[1] + vexact_bar(q64, kb, vx))
            assert ok, (q_scale, b, err)


@pytest.mark.parametrize("where", ["k_scale_inf", "k_min_nan", "v_scale_inf", "v_min_nan", "k_alpha_nan", "v_alpha_nan"])
def test_default_path_flags_nonfinite_metadata(where):
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    rng = np.random.default_rng(13)
    cache = new_cache(1, 2, 8, 8, torch.float16)
    fill(cache, 0, workloads.np_kv(rng, (2, 64 * 6 + 7, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32),
         workloads.np_kv(rng, (2, 64 * 6 + 7, 128), (), 0.5).astype(np.float32))
    page = int(cache.block_table[0, 3])
    pool, key, val = {"k_scale_inf": (cache.k_pool, "scale", float("inf")),
                      "k_min_nan": (cache.k_pool, "min", float("nan")),
                      "v_scale_inf": (cache.v_pool, "scale", float("inf")),
                      "v_min_nan": (cache.v_pool, "min", float("nan")),
                      "k_alpha_nan": (cache.k_pool, "alpha", float("nan")),
                      "v_alpha_nan": (cache.v_pool, "alpha", float("nan"))}[where]
    pool[key][1, page, 17] = val
    q = (rng.standard_normal((1, 8, 128)) / np.sqrt(128)).astype(np.float16)
    cache.attend(torch.from_numpy(q).cuda())
    with pytest.raises(w.NumericalFailure):
        cache.check()


@pytest.mark.parametrize("mode", ["k", "exact"])
def test_sequence_without_tokens(mode):
    """A sequence with neither sealed blocks nor tail rows beside two others: its outputs are
    the merge of zero partials (0 / 0, flagged as non-finite), the others' match the bridge
    (small batch: the merge runs fused in the chunk kernels)."""
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    rng = np.random.default_rng(17)
    h, hq, lens = 2, 8, [0, 64 * 3 + 9, 64 * 2]
    cache = new_cache(len(lens), h, hq, 4, torch.float16, mode)
    srcs = []
    for b, L in enumerate(lens):
        k = workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32)
        v = workloads.np_kv(rng, (h, L, 128), (), 0.5).astype(np.float32)
        if L:
            fill(cache, b, k, v)
        srcs.append((k, v))
    q = (rng.standard_normal((len(lens), hq, 128)) / np.sqrt(128)).astype(np.float16)
    out = cache.attend(torch.from_numpy(q).cuda()).float().cpu().numpy()
    assert np.isnan(out[0]).all()
    with pytest.raises(w.NumericalFailure):
        cache.check()
    for b in (1, 2):
        k, v = srcs[b]
        nb = lens[b] // 64
        kb, vb = rows(k, nb, "float16", "bridge"), rows(v, nb, "float16", "bridge")
        ok, err = O.within_tolerance(out[b], attention64(q[b].astype(np.float64), kb, vb), *O.TOLERANCE["float16"])
        assert ok, (b, err)


def test_cfg1_full_size_default_path():
    """cfg1: one 32768-token sequence, 511 sealed INT3 blocks + a 64-token native tail, 32:8."""
    from nsn_b200 import workloads
    k, v, q, nb, t = workloads.np_config(1)
    assert (nb, t) == (511, 64)
    k, v = k[0].astype(np.float32), v[0].astype(np.float32)
    q = q.reshape(1, 32, 128).astype(np.float32)
    cache = new_cache(1, 8, 32, 512, torch.float16)
    extra = fill(cache, 0, k, v, tail64=True)
    assert int(cache.n_blocks[0]) == 511 and int(cache.tail_len[0]) == 63
    out32 = torch.empty((1, 32, 128), dtype=torch.float32, device="cuda")
    out = cache.attend(torch.from_numpy(q).cuda().half(), *extra, out_f32=out32)
    cache.check()
    q64 = q[0].astype(np.float64)
    rk, rv = Restored(k, nb, "float16"), Restored(v, nb, "float16")
    T = k.shape[1]
    kb, vb, vx = rk.rows(T, nb, "bridge"), rv.rows(T, nb, "bridge"), rv.rows(T, nb, "exact")
    ok, err = O.within_tolerance(out[0].float().cpu().numpy(), attention64(q64, kb, vb), *O.TOLERANCE["float16"])
    assert ok, err
    ok, err = O.within_tolerance(out32[0].cpu().numpy(), attention64(q64, kb, vx), KROUND[0],
                                 KROUND[1] + vexact_bar(q64, kb, vx))
    assert ok, err


@pytest.mark.parametrize("mode", ["k", "exact"])
def test_cfg2_full_bench_state(mode):
    """The benchmark's cfg2 state: 64 sequences of U{32..256} blocks + U[0,63] tails, 32:8,
    then 64 decode steps (append one token per sequence, attend, seal full tails).  A sample
    of sequences is checked against the fp64 oracle at three steps: against the bridge at
    the parity bar in both modes, and against the mode's own arithmetic (K rounded / exact,
    V exact) at the tight bar."""
    from nsn_b200 import workloads
    c = workloads.CONFIGS[2]
    blocks, tails = workloads.np_cfg2_lengths()
    B, h, hq = c["batch"], c["h"], c["hq"]
    steps = 64
    cache = new_cache(B, h, hq, int(blocks.max()) + 2, torch.float16, mode)
    gen = torch.Generator(device="cuda").manual_seed(2)
    sample = (0, 17, 42, 63)
    host, new_k, new_v = {}, [], []
    for b in range(B):
        L = int(blocks[b]) * 64 + int(tails[b])
        kk = workloads.torch_kv(gen, (h, L + steps, 128), c["k_outliers"], 0.5)
        vv = workloads.torch_kv(gen, (h, L + steps, 128), (), c["v_sigma"])
        cache.prefill(b, kk[:, :L], vv[:, :L])
        if b in sample:
            k, v = kk.float().cpu().numpy(), vv.float().cpu().numpy()
            nb_last = (L + steps - 1) // 64
            host[b] = (L, Restored(k, nb_last, "float16"), Restored(v, nb_last, "float16"))
        new_k.append(kk[:, L:])
        new_v.append(vv[:, L:])
    new_k, new_v = torch.stack(new_k), torch.stack(new_v)  # [B, h, steps, 128]
    qs = (torch.randn((steps, B, hq, 128), generator=gen, device="cuda") / np.sqrt(128)).half()
    check_at = (0, 31, 63)
    outs = {}
    out32 = torch.empty((B, hq, 128), dtype=torch.float32, device="cuda")
    seals = 0
    for s in range(steps):
        if s in check_at:  # the fp32 context over the history, before this step's append
            cache.attend(qs[s], out_f32=out32)
            ctx = out32.cpu().numpy().copy()
        before = cache.n_blocks.clone()
        o = cache.step(qs[s], new_k[:, :, s].contiguous(), new_v[:, :, s].contiguous())  # nsnkv_paged_step
        seals += int((cache.n_blocks - before).sum())
        if s in check_at:
            outs[s] = (o.float().cpu().numpy(), ctx)
    cache.check()
    assert seals == B  # every tail of 0..63 tokens reaches 64 exactly once in 64 appends
    for b in sample:
        L0, rk, rv = host[b]
        for s in check_at:
            q64 = qs[s, b].float().cpu().numpy().astype(np.float64)
            got, got32 = outs[s]
            # the step's output: the history plus this step's token, blocks sealed before it
            T = L0 + s + 1
            nb = (T - 1) // 64
            kb, vb = rk.rows(T, nb, "bridge"), rv.rows(T, nb, "bridge")
            ok, err = O.within_tolerance(got[b], attention64(q64, kb, vb), *O.TOLERANCE["float16"])
            assert ok, ("bridge", mode, b, s, err)
            # the context before the append, against the mode's own arithmetic
            T = L0 + s
            nb = T // 64
            vx = rv.rows(T, nb, "exact")
            kk = rk.rows(T, nb, "bridge" if mode == "k" else "exact")
            bar = vexact_bar(q64, kk, vx) + (exact_k_bar(q64, kk, vx) if mode == "exact" else 0.0)
            ok, err = O.within_tolerance(got32[b], attention64(q64, kk, vx), KROUND[0], KROUND[1] + bar)
            assert ok, ("own arithmetic", mode, b, s, err)


def test_two_streams_get_separate_workspaces():
    """decode_attention without ws= on two streams at once: each stream has its own split-KV
    workspace, so both outputs match the oracle (a shared buffer would race on the partials)."""
    from nsn_b200 import workloads
    from nsn_b200.kernel import decode_attention
    rng = np.random.default_rng(77)
    caches, hist, qs = [], [], []
    for _ in range(2):
        lens = [64 * 40 + 5, 64 * 37 + 60]
        c = new_cache(2, 2, 8, 41, torch.float16)
        hk = [workloads.np_kv(rng, (2, L, 128), workloads.K_OUTLIERS_4, 0.5).astype(np.float32) for L in lens]
        hv = [workloads.np_kv(rng, (2, L, 128), (), 0.5).astype(np.float32) for L in lens]
        for b in range(2):
            fill(c, b, hk[b], hv[b])
        caches.append(c)
        hist.append((lens, hk, hv))
        qs.append(torch.from_numpy((rng.standard_normal((2, 8, 128)) / np.sqrt(128)).astype(np.float16)).cuda())
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = []
    for c, q, st in zip(caches, qs, streams):
        with torch.cuda.stream(st):
            o = torch.empty((2, 8, 128), dtype=torch.float16, device="cuda")
            for _ in range(20):  # repeated calls keep the two streams' kernels overlapping
                decode_attention(q, c.k_pool, c.v_pool, h=2, bits=3, blk_stride_head=c.pages, blk_stride_page=1,
                                 n_blocks=c.n_blocks, max_blocks=c.max_blocks, k_tail=c.k_tail, v_tail=c.v_tail,
                                 tail_stride_seq=2 * 64, tail_stride_head=64, tail_len=c.tail_len, max_tail=63,
                                 block_table=c.block_table, out=o, status=c.status)
            outs.append(o)
    torch.cuda.synchronize()
    for c, (lens, hk, hv), q, o in zip(caches, hist, qs, outs):
        c.check()
        for b, L in enumerate(lens):
            nb = L // 64
            want = attention64(q[b].float().cpu().numpy().astype(np.float64), rows(hk[b], nb, "float16", "bridge"),
                               rows(hv[b], nb, "float16", "bridge"))
            ok, err = O.within_tolerance(o[b].float().cpu().numpy(), want, *O.TOLERANCE["float16"])
            assert ok, (b, err)
