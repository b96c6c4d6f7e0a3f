"""GPU tests of the renorm-factor path (nsnkv_block_renorm, nsnkv_seal_full_tails_alpha,
nsnkv_decode_attn_alpha) in its exact mode.

* alpha = n / max(||min + scale * code||, 1e-12) per token against the oracle's decode.
* Attention through a paged cache built with restore_rounding="exact" (sealed blocks on
  attn_sealed3_kernel, tails on attn_native_rows_kernel) against fp64 attention over
  the exact fp32 restore of the same blocks (nsn_decode without the final cast), with a
  tight bar, and against the reference bridge (rows rounded to fp16) with the parity bar.
* GQA groups 1..4, q magnitudes that need the exponent shift, zero-norm tokens,
  constant blocks, chunk sizes that leave warps idle, appended tokens and seals.
The default mode (K rounded like the bridge) is tested in test_gpu_sealed.py.
"""
import numpy as np
import pytest
import torch

from oracle import nsn_oracle as O

pytestmark = pytest.mark.gpu

TIGHT = (1e-4, 2e-5)  # (rtol, atol) against the exact fp32 restore: fp32 accumulation only


def mma_bar(q, k, v):
    """Extra absolute bar for the tensor-core dot products over codes.

    The K codes enter mma.sync as fp16 subnormals, whose sums the tensor core keeps to
    less than fp32 precision.  The bar allows each logit an error of 2^-16 * sum_c |q_c k_c|
    / sqrt(128), which moves an output by at most that times max |v|; every case in this
    file stays inside it.  With 1/sqrt(128)-scaled queries the bar is about 1e-5."""
    rep = q.shape[0] // k.shape[0]
    sabs = np.einsum("jd,jtd->jt", np.abs(q), np.abs(np.repeat(k, rep, 0))).max() / np.sqrt(128.0)
    return 2.0 ** -16 * sabs * np.abs(v).max()


def exact_restore(q8, n16, m16, s16):
    """nsn_decode (loop_kv_nb06_primitives.py:57-66) in fp64, without the cast to fp16."""
    d = m16.astype(np.float64) + s16.astype(np.float64) * q8.astype(np.float64)
    den = np.maximum(np.sqrt((d * d).sum(-1, keepdims=True)), 1e-12)
    n = n16.astype(np.float64)
    return np.where(n == 0, 0.0, n * d / den)


def attention64(q, k, v):
    """q [hq,128], k/v [h,T,128] fp64 -> [hq,128] (repeat_kv grouping, scale 1/sqrt(128))."""
    h = k.shape[0]
    rep = q.shape[0] // h
    out = np.empty((q.shape[0], 128))
    for j in range(q.shape[0]):
        s = k[j // rep] @ q[j] / np.sqrt(128.0)
        p = np.exp(s - s.max())
        out[j] = (p[:, None] * v[j // rep]).sum(0) / p.sum()
    return out


def history_oracle(hk, hv, nb, rows="exact"):
    """Full K/V [h,T,128] in fp64: nb sealed blocks restored (exactly, or as the bridge's fp16 rows) + the tail."""
    parts_k, parts_v = [], []
    for src, parts in ((hk, parts_k), (hv, parts_v)):
        h = src.shape[0]
        if nb:
            x = src[None, :, :nb * 64].astype(np.float32).reshape(1, h, nb, 64, 128)
            q8, n, m, s, st = O.nsn_encode(x, 3)
            assert st == 0
            if rows == "exact":
                y = exact_restore(q8, n, m, s)
            else:
                y = np.asarray(O.nsn_decode(q8, n, m, s, "float16"), np.float64)
            parts.append(y.reshape(h, nb * 64, 128))
        parts.append(src[:, nb * 64:].astype(np.float64))
    return np.concatenate(parts_k, 1), np.concatenate(parts_v, 1)


def make_cache(rng, lens, h, hq, max_blocks, q_scale=1.0, mode="exact"):
    from nsn_b200 import workloads
    from nsn_b200.paged import PagedKVCache
    hk = [workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5) for L in lens]
    hv = [workloads.np_kv(rng, (h, L, 128), (), 0.5) for L in lens]
    cache = PagedKVCache(len(lens), h, max_blocks=max_blocks, bits=3, dtype=torch.float16, hq=hq,
                         restore_rounding=mode)
    for b in range(len(lens)):
        cache.prefill(b, torch.from_numpy(hk[b]).cuda(), torch.from_numpy(hv[b]).cuda())
    q = (rng.standard_normal((len(lens), hq, 128)) * q_scale / np.sqrt(128)).astype(np.float16)
    return cache, hk, hv, q


@pytest.mark.parametrize("bits", [3, 4, 5])
def test_block_renorm_matches_oracle(bits):
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    rng = np.random.default_rng(bits)
    x = workloads.np_kv(rng, (3, 5, 64, 128), workloads.K_OUTLIERS_4, 0.5)
    x[0, 1, 7] = 0.0  # a zero-norm token
    x[1, 2] = 0.25    # a constant block (all codes 0, scale 0)
    xt = torch.from_numpy(x).cuda()
    pool = dict(codes=torch.zeros((3, 7, w.code_bytes(bits)), dtype=torch.uint8, device="cuda"),
                norm=torch.zeros((3, 7, 64), dtype=torch.float16, device="cuda"),
                min=torch.zeros((3, 7, 128), dtype=torch.float16, device="cuda"),
                scale=torch.zeros((3, 7, 128), dtype=torch.float16, device="cuda"),
                alpha=torch.full((3, 7, 64), -1.0, dtype=torch.float32, device="cuda"))
    w.encode_blocks(xt, bits, out=pool, out_row_stride=7, out_offset=1, check=False)
    q8, n, m, s, st = O.nsn_encode(x.astype(np.float32), bits)
    d = m.astype(np.float64) + s.astype(np.float64) * q8.astype(np.float64)
    den = np.maximum(np.sqrt((d * d).sum(-1)), 1e-12)
    n64 = n[..., 0].astype(np.float64)
    want = np.where(n64 == 0, 0.0, n64 / den)
    got = pool["alpha"].cpu().numpy()
    assert np.all(got[:, 0] == -1.0) and np.all(got[:, 6] == -1.0), "wrote outside the encoded blocks"
    np.testing.assert_allclose(got[:, 1:6], want, rtol=2e-6, atol=0)
    assert np.all(got[0, 2, 7] == 0.0)


@pytest.mark.parametrize("h,hq", [(2, 8), (2, 6), (4, 8), (3, 3)])
def test_alpha_path_tight_against_exact_restore(h, hq):
    rng = np.random.default_rng(100 + hq)
    lens = [64, 1, 130, 64 * 9 + 17, 64 * 21, 64 * 5 + 63]
    cache, hk, hv, q = make_cache(rng, lens, h, hq, max_blocks=22)
    assert cache.uses_alpha_path()
    out32 = torch.empty((len(lens), hq, 128), dtype=torch.float32, device="cuda")
    out = cache.attend(torch.from_numpy(q).cuda(), out_f32=out32)
    cache.check()
    got32, got16 = out32.cpu().numpy(), out.float().cpu().numpy()
    for b, L in enumerate(lens):
        nb = L // 64
        k, v = history_oracle(hk[b], hv[b], nb, "exact")
        q64 = q[b].astype(np.float64)
        want = attention64(q64, k, v)
        ok, err = O.within_tolerance(got32[b], want, TIGHT[0], TIGHT[1] + mma_bar(q64, k, v))
        assert ok, (b, L, err)
        kb, vb = history_oracle(hk[b], hv[b], nb, "bridge")
        ok, err = O.within_tolerance(got16[b], attention64(q[b].astype(np.float64), kb, vb), *O.TOLERANCE["float16"])
        assert ok, (b, L, err)


@pytest.mark.parametrize("q_scale", [1e-3, float(np.sqrt(128)), 300.0, 4000.0])
def test_alpha_path_q_magnitudes(q_scale):
    """q far from unit scale: tiny values and values whose q * 2^7 leaves the fp16 range.

    The bar adds the tensor-core bound of mma_bar, which grows with |q|."""
    rng = np.random.default_rng(7)
    lens = [64 * 12 + 5, 64 * 4]
    cache, hk, hv, q = make_cache(rng, lens, 2, 8, max_blocks=13, q_scale=q_scale)
    out32 = torch.empty((len(lens), 8, 128), dtype=torch.float32, device="cuda")
    cache.attend(torch.from_numpy(q).cuda(), out_f32=out32)
    cache.check()
    for b, L in enumerate(lens):
        k, v = history_oracle(hk[b], hv[b], L // 64, "exact")
        q64 = q[b].astype(np.float64)
        want = attention64(q64, k, v)
        bar = mma_bar(q64, k, v)
        ok, err = O.within_tolerance(out32[b].cpu().numpy(), want, TIGHT[0], TIGHT[1] + bar)
        assert ok, (q_scale, b, err, bar)


def test_alpha_path_zero_and_constant_blocks():
    from nsn_b200 import workloads
    from nsn_b200.paged import PagedKVCache
    rng = np.random.default_rng(3)
    h, hq, L = 2, 8, 64 * 6 + 9
    hk = workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5)
    hv = workloads.np_kv(rng, (h, L, 128), (), 0.5)
    hk[:, 64:128] = 0.0          # a zero K block: every norm 0
    hv[0, 128:192] = 0.5         # a constant V block: scale 0
    hk[1, 200:203] = 0.0         # zero-norm tokens inside a block
    hv[1, 300] = 0.0
    cache = PagedKVCache(1, h, max_blocks=8, bits=3, dtype=torch.float16, hq=hq, restore_rounding="exact")
    cache.prefill(0, torch.from_numpy(hk).cuda(), torch.from_numpy(hv).cuda())
    q = (rng.standard_normal((1, hq, 128)) / np.sqrt(128)).astype(np.float16)
    out32 = torch.empty((1, hq, 128), dtype=torch.float32, device="cuda")
    cache.attend(torch.from_numpy(q).cuda(), out_f32=out32)
    cache.check()
    k, v = history_oracle(hk, hv, L // 64, "exact")
    q64 = q[0].astype(np.float64)
    ok, err = O.within_tolerance(out32[0].cpu().numpy(), attention64(q64, k, v), TIGHT[0],
                                 TIGHT[1] + mma_bar(q64, k, v))
    assert ok, err


def test_alpha_path_agrees_with_restore_path():
    """The same cache attended through nsnkv_decode_attn (norms, bridge rounding) and the exact renorm-factor kernel."""
    from nsn_b200.kernel import decode_attention
    from nsn_b200 import primitives as w
    rng = np.random.default_rng(11)
    lens = [64 * 30 + 3, 64 * 7, 64 * 16 + 40]
    cache, hk, hv, q = make_cache(rng, lens, 2, 8, max_blocks=31)
    qt = torch.from_numpy(q).cuda()
    fast = cache.attend(qt).float().cpu().numpy()
    # the restore path reads the reference's code order: dense copies, V rows unpaired
    pools = [{k: p[k].contiguous() for k in ("codes", "norm", "min", "scale")} for p in (cache.k_pool, cache.v_pool)]
    for p_, src in zip(pools, (cache.k_pool, cache.v_pool)):
        p_["codes"] = w.from_code_order(p_["codes"], 3, src["code_order"])
    slow, st = decode_attention(
        qt, pools[0], pools[1], h=cache.h, bits=3, blk_stride_head=cache.pages, blk_stride_page=1,
        n_blocks=cache.n_blocks, max_blocks=cache.max_blocks, k_tail=cache.k_tail, v_tail=cache.v_tail,
        tail_stride_seq=cache.h * w.BLOCK, tail_stride_head=w.BLOCK, tail_len=cache.tail_len, max_tail=w.BLOCK - 1,
        block_table=cache.block_table)
    assert int(st.item()) == 0
    ok, err = O.within_tolerance(fast, slow.float().cpu().numpy(), *O.TOLERANCE["float16"])
    assert ok, err


def test_seal_writes_renorm_factors():
    """After decode steps that seal pages, every sealed page's alpha equals nsnkv_block_renorm's."""
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    rng = np.random.default_rng(5)
    lens = [60, 120, 64]
    cache, hk, hv, q = make_cache(rng, lens, 2, 8, max_blocks=4)
    for s in range(70):
        qq = (rng.standard_normal((3, 8, 128)) / np.sqrt(128)).astype(np.float16)
        kn = workloads.np_kv(rng, (3, 2, 1, 128), workloads.K_OUTLIERS_4, 0.5)[:, :, 0]
        vn = workloads.np_kv(rng, (3, 2, 1, 128), (), 0.5)[:, :, 0]
        cache.step(torch.from_numpy(qq).cuda(), torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
    cache.check()
    nb = cache.n_blocks.cpu().tolist()
    assert nb == [(L + 70) // 64 for L in lens]
    for pool in (cache.k_pool, cache.v_pool):
        sealed = pool["alpha"].clone()
        pool["alpha"].fill_(-1.0)
        for b in range(3):
            w.block_renorm(pool, 3, cache.h, nb[b], cache.pages, b * cache.max_blocks)
        torch.cuda.synchronize()
        for b in range(3):
            pages = cache.block_table[b, :nb[b]].long()
            assert torch.equal(sealed[:, pages], pool["alpha"][:, pages]), b


def test_bridge_rounding_option_matches_bridge_on_unscaled_queries():
    """cfg0-style queries (N(0,1), not scaled by 1/sqrt(128)): the bridge's fp16 rounding of
    restored rows alone moves outputs past the parity bar, so a cache built with
    restore_rounding="kv" (restore kernel, rows rounded like restore_group) matches the
    bridge there, and the exact mode matches the exact restore."""
    lens = [64 * 15 + 3, 64 * 8]
    for bridge in (True, False):
        r = np.random.default_rng(9)
        cache, hk, hv, q = make_cache(r, lens, 2, 8, max_blocks=16, q_scale=float(np.sqrt(128)),
                                      mode="kv" if bridge else "exact")
        assert cache.uses_alpha_path() == (not bridge)
        out32 = torch.empty((len(lens), 8, 128), dtype=torch.float32, device="cuda")
        out = cache.attend(torch.from_numpy(q).cuda(), out_f32=out32)
        cache.check()
        for b, L in enumerate(lens):
            q64 = q[b].astype(np.float64)
            if bridge:
                kb, vb = history_oracle(hk[b], hv[b], L // 64, "bridge")
                ok, err = O.within_tolerance(out[b].float().cpu().numpy(), attention64(q64, kb, vb),
                                             *O.TOLERANCE["float16"])
            else:
                k, v = history_oracle(hk[b], hv[b], L // 64, "exact")
                ok, err = O.within_tolerance(out32[b].cpu().numpy(), attention64(q64, k, v), TIGHT[0],
                                             TIGHT[1] + mma_bar(q64, k, v))
            assert ok, (bridge, b, err)


@pytest.mark.parametrize("where", ["k_scale_inf", "k_min_nan", "v_scale_inf", "v_min_nan", "alpha_nan"])
def test_alpha_path_flags_nonfinite_metadata(where):
    """A non-finite value in a sealed block's metadata surfaces as NumericalFailure from check()."""
    from nsn_b200 import primitives as w
    rng = np.random.default_rng(13)
    cache, hk, hv, q = make_cache(rng, [64 * 6 + 7], 2, 8, max_blocks=8)
    page = int(cache.block_table[0, 3])
    pool, key, val = {"k_scale_inf": (cache.k_pool, "scale", float("inf")),
                      "k_min_nan": (cache.k_pool, "min", float("nan")),
                      "v_scale_inf": (cache.v_pool, "scale", float("inf")),
                      "v_min_nan": (cache.v_pool, "min", float("nan")),
                      "alpha_nan": (cache.v_pool, "alpha", float("nan"))}[where]
    pool[key][1, page, 17] = val
    cache.attend(torch.from_numpy(q).cuda())
    with pytest.raises(w.NumericalFailure):
        cache.check()


def test_block_records_match_dense_arrays():
    """The cache's block records (one copy per block, K codes as paired halves, V codes as
    paired rows) and dense copies of the same arrays in the reference's order (eight copies
    per block) agree within fp32 accumulation order; records with codes in the reference's
    order on the restore path match dense arrays bit for bit."""
    from nsn_b200.kernel import decode_attention
    from nsn_b200 import primitives as w
    rng = np.random.default_rng(21)
    lens = [64 * 40 + 9, 64 * 3, 64 * 77 + 63, 5]
    cache, hk, hv, q = make_cache(rng, lens, 2, 8, max_blocks=80)
    assert cache.blk_bytes == 7680 and w.blk_bytes_of(cache.k_pool, 3) == 7680
    assert cache.k_pool["code_order"] == 2 and cache.v_pool["code_order"] == 1
    qt = torch.from_numpy(q).cuda()
    common = dict(h=cache.h, bits=3, blk_stride_head=cache.pages, blk_stride_page=1, n_blocks=cache.n_blocks,
                  max_blocks=cache.max_blocks, k_tail=cache.k_tail, v_tail=cache.v_tail,
                  tail_stride_seq=cache.h * w.BLOCK, tail_stride_head=w.BLOCK, tail_len=cache.tail_len,
                  max_tail=w.BLOCK - 1, block_table=cache.block_table)

    def dense_of(keys):
        d = [{k: p[k].contiguous() for k in keys} for p in (cache.k_pool, cache.v_pool)]
        for p_, src in zip(d, (cache.k_pool, cache.v_pool)):
            p_["codes"] = w.from_code_order(p_["codes"], 3, src["code_order"])
        return d

    # renorm-factor path: records (paired halves / rows) against dense arrays: the K codes
    # enter the tensor cores in another k order, so fp32 sums may round differently
    keys = ("codes", "norm", "min", "scale", "alpha")
    dense = dense_of(keys)
    assert w.blk_bytes_of(dense[0], 3) == 0
    fa = torch.empty(q.shape, device="cuda")
    fb = torch.empty(q.shape, device="cuda")
    a, sa = decode_attention(qt, cache.k_pool, cache.v_pool, out_f32=fa, exact=True, **common)
    b, sb = decode_attention(qt, dense[0], dense[1], out_f32=fb, exact=True, **common)
    torch.cuda.synchronize()
    assert int(sa.item()) == 0 and int(sb.item()) == 0
    assert torch.allclose(fa, fb, rtol=TIGHT[0], atol=TIGHT[1]), (fa - fb).abs().max().item()
    # restore path: the same record strides with V rows back in the reference's order
    from nsn_b200.paged import block_record_pools
    rec, kp, vp = block_record_pools(cache.h, cache.pages, 3, "cuda")
    rec.copy_(cache.records)
    for p_ in (kp, vp):
        p_["codes"].copy_(w.from_code_order(p_["codes"], 3, p_.pop("code_order")))
    keys = ("codes", "norm", "min", "scale")
    for p_, src in ((kp, cache.k_pool), (vp, cache.v_pool)):
        p_["norm"].copy_(src["norm"])
    dense = dense_of(keys)
    a, sa = decode_attention(qt, {k: kp[k] for k in keys}, {k: vp[k] for k in keys}, **common)
    b, sb = decode_attention(qt, dense[0], dense[1], **common)
    torch.cuda.synchronize()
    assert int(sa.item()) == 0 and int(sb.item()) == 0
    assert torch.equal(a, b)
    # paired V rows without factors have no kernel
    with pytest.raises(w.ContractError):
        decode_attention(qt, {k: cache.k_pool[k] for k in keys}, dict({k: cache.v_pool[k] for k in keys}, code_order=1),
                         **common)


def test_encode_into_block_records_matches_dense():
    """encode_blocks into record views writes the dense encoder's bytes, and the factors
    nsnkv_block_renorm writes there equal the dense ones."""
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    from nsn_b200.paged import block_record_pools
    rng = np.random.default_rng(22)
    x = torch.from_numpy(workloads.np_kv(rng, (2, 6, 64, 128), workloads.K_OUTLIERS_4, 0.5)).cuda()
    rec, kp, _ = block_record_pools(2, 9, 3, "cuda")
    w.encode_blocks(x, 3, out=kp, out_row_stride=9, out_offset=2)
    ref = w.encode_blocks(x, 3)
    dense = dict(codes=ref["codes"], norm=ref["metas"][0].reshape(2, 6, 64), min=ref["metas"][1].reshape(2, 6, 128),
                 scale=ref["metas"][2].reshape(2, 6, 128), alpha=torch.zeros((2, 6, 64), device="cuda"))
    w.block_renorm(dense, 3, 2, 6, 6)
    torch.cuda.synchronize()
    for k in ("codes", "norm", "min", "scale", "alpha"):
        got = kp[k][:, 2:8]
        if k == "codes":  # the records keep K codes as paired halves
            got = w.from_code_order(got, 3, kp["code_order"])
        assert torch.equal(got, dense[k]), k
    assert int(rec[:, :2].count_nonzero()) == 0 and int(rec[:, 8:].count_nonzero()) == 0


@pytest.mark.parametrize("bits", [3, 5])
@pytest.mark.parametrize("order", [1, 2])
def test_code_orders_encode_and_renorm(bits, order):
    """Encoding into a pool with code_order 1 (paired rows) or 2 (paired halves) writes that
    order of the dense encoder's codes, and nsnkv_block_renorm reading it gives the dense
    factors (generic and fp16 encoders)."""
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    rng = np.random.default_rng(23 + bits)
    for dtype in (torch.float16, torch.bfloat16):
        x = torch.from_numpy(workloads.np_kv(rng, (3, 4, 64, 128), (), 0.5)).cuda().to(dtype)
        pool = dict(codes=torch.zeros((3, 6, w.code_bytes(bits)), dtype=torch.uint8, device="cuda"),
                    norm=torch.zeros((3, 6, 64), dtype=torch.float16, device="cuda"),
                    min=torch.zeros((3, 6, 128), dtype=torch.float16, device="cuda"),
                    scale=torch.zeros((3, 6, 128), dtype=torch.float16, device="cuda"),
                    alpha=torch.zeros((3, 6, 64), dtype=torch.float32, device="cuda"), code_order=order)
        w.encode_blocks(x, bits, out=pool, out_row_stride=6, out_offset=1)
        ref = w.encode_blocks(x, bits)
        dense = dict(codes=ref["codes"], norm=ref["metas"][0].reshape(3, 4, 64), min=ref["metas"][1].reshape(3, 4, 128),
                     scale=ref["metas"][2].reshape(3, 4, 128), alpha=torch.zeros((3, 4, 64), device="cuda"))
        w.block_renorm(dense, bits, 3, 4, 4)
        torch.cuda.synchronize()
        assert torch.equal(pool["codes"][:, 1:5], w.to_code_order(dense["codes"], bits, order)), dtype
        assert torch.equal(pool["alpha"][:, 1:5], dense["alpha"]), dtype
        assert torch.equal(w.from_code_order(pool["codes"][:, 1:5], bits, order), dense["codes"]), dtype
