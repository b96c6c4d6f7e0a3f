"""GPU tests of the cache paths and the split-KV merge.

* PackedCache (the reference's per-slot policy) against the state the reference's
  own PackedCache reached on the same inputs (tests/golden, bit for bit).
* PagedKVCache (batched, seal-at-64): every step's output against the fp64 oracle
  over the sequence's history, and every sealed page against the oracle's encode.
* Split-KV: per-shard partials merged by nsnkv_merge_shards equal one-pass attention.
"""
import hashlib

import numpy as np
import pytest
import torch

import golden_util as G
from oracle import nsn_oracle as O

pytestmark = pytest.mark.gpu


def bits16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class FixtureBase:
    """Minimal stand-in for the HF DynamicCache surface PackedCache uses."""

    def __init__(self):
        self.key_cache = []
        self.value_cache = []
        self._seen_tokens = 0

    def get_seq_length(self, layer_idx=0):
        if layer_idx >= len(self.key_cache) or self.key_cache[layer_idx] is None:
            return 0
        return self.key_cache[layer_idx].shape[-2]

    def update(self, k, v, i, cache_kwargs=None):
        while len(self.key_cache) <= i:
            self.key_cache.append(None)
            self.value_cache.append(None)
        for data, x in ((self.key_cache, k), (self.value_cache, v)):
            data[i] = x if data[i] is None else torch.cat((data[i], x), -2)
        return self.key_cache[i], self.value_cache[i]


def test_packed_cache_lifecycle_matches_reference():
    from nsn_b200 import primitives as w
    from nsn_b200.packed import make_packed_cache
    idx = G.index()["cache"]
    gen = torch.Generator(device="cpu").manual_seed(2026093001 + 7)
    x_cpu = torch.randn(idx["slots"], 2, idx["last"], 128, generator=gen).to(torch.bfloat16)
    assert G.matches("cache_x", bits16(x_cpu))
    x = x_cpu.cuda()
    old = (w.LAYERS, w.HEADS)
    try:
        w.LAYERS, w.HEADS = 2, 2
        cache = make_packed_cache(FixtureBase)(1, 3)
        prefill = idx["prefill"]
        for end in [prefill] + list(range(prefill + 1, idx["last"] + 1)):
            start = 0 if end == prefill else end - 1
            for s in range(idx["slots"]):
                k = x[s:s + 1, :, start:end, :]
                v = (k.float() * .75).to(torch.bfloat16)
                rk, rv = cache.update(k, v, s, {"cache_position": torch.arange(start, end, device="cuda")})
                if end in idx["checkpoints"]:
                    assert G.matches(f"cache_ret_{end}_{s}_k", bits16(rk)), (end, s)
                    assert G.matches(f"cache_ret_{end}_{s}_v", bits16(rv)), (end, s)
            if end == prefill:
                cache.post_prefill()
            else:
                cache.post_decode()
        assert cache.compressed.get(0, 0) == idx["final_compressed"]
        for s in range(idx["slots"]):
            for kv in ("K", "V"):
                g = cache.packed[(s, kv)]
                assert G.matches(f"cache_final_{s}_{kv}_codes", g["codes"].cpu().numpy())
                assert G.matches(f"cache_final_{s}_{kv}_headers", g["headers"].cpu().numpy())
                for tag, m in zip("nms", g["metas"]):
                    assert G.matches(f"cache_final_{s}_{kv}_{tag}", bits16(m))
                tail = (cache.key_cache if kv == "K" else cache.value_cache)[s]
                assert G.matches(f"cache_final_{s}_{kv}_tail", bits16(tail))
        cache.clear()
        assert not cache.packed and not cache.key_cache
    finally:
        w.LAYERS, w.HEADS = old


def _oracle_step(hist_k, hist_v, q, bits=3):
    """fp64 attention of q [hq,128] over one sequence's history [h,L,128] (fp16 values),
    with floor((L-1)/64) blocks sealed (the appended token is always native)."""
    h, L = hist_k.shape[0], hist_k.shape[1]
    nb = (L - 1) // 64
    fulls = []
    for src in (hist_k, hist_v):
        src = src[None].astype(np.float32)
        if nb:
            qq, n, m, s, st = O.nsn_encode(src[:, :, :nb * 64].reshape(1, h, nb, 64, 128), bits)
            assert st == 0
            fulls.append(O.restore_full(qq, n, m, s, src[:, :, nb * 64:], "float16"))
        else:
            fulls.append(src)
    out, _ = O.bridge_attention(q[None, :, None, :].astype(np.float32), fulls[0], fulls[1])
    return out[0]


def test_paged_cache_steps_and_seals():
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    from nsn_b200.paged import PagedKVCache
    rng = np.random.default_rng(21)
    h, hq, steps = 2, 8, 70
    lens = [100, 250, 127, 64]
    hist_k = [workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5) for L in lens]
    hist_v = [workloads.np_kv(rng, (h, L, 128), (), 0.5) for L in lens]
    cache = PagedKVCache(len(lens), h, max_blocks=8, bits=3, dtype=torch.float16, hq=hq)
    for b in range(len(lens)):
        cache.prefill(b, torch.from_numpy(hist_k[b]).cuda(), torch.from_numpy(hist_v[b]).cuda())
    check_at = {0, 1, 13, 27, 28, 29, 36, 37, 60, 69}
    for s in range(steps):
        q = (rng.standard_normal((len(lens), hq, 128)) / np.sqrt(128)).astype(np.float16)
        kn = workloads.np_kv(rng, (len(lens), h, 1, 128), workloads.K_OUTLIERS_4, 0.5)[:, :, 0]
        vn = workloads.np_kv(rng, (len(lens), h, 1, 128), (), 0.5)[:, :, 0]
        out = cache.step(torch.from_numpy(q).cuda(), torch.from_numpy(kn).cuda(), torch.from_numpy(vn).cuda())
        for b in range(len(lens)):
            hist_k[b] = np.concatenate([hist_k[b], kn[b][:, None]], 1)
            hist_v[b] = np.concatenate([hist_v[b], vn[b][:, None]], 1)
        if s in check_at:
            got = out.float().cpu().numpy()
            for b in range(len(lens)):
                want = _oracle_step(hist_k[b], hist_v[b], q[b])
                ok, err = O.within_tolerance(got[b], want, *O.TOLERANCE["float16"])
                assert ok, (s, b, err)
    cache.check()
    lengths = cache.lengths().tolist()
    assert lengths == [L + steps for L in lens]
    nb = cache.n_blocks.cpu().tolist()
    assert nb == [(L + steps) // 64 for L in lens]
    assert cache.tail_len.cpu().tolist() == [(L + steps) % 64 for L in lens]
    # every sealed page equals the oracle's encode of that 64-token window
    for b in range(len(lens)):
        for kv, hist, pool in (("K", hist_k, cache.k_pool), ("V", hist_v, cache.v_pool)):
            x = hist[b][:, :nb[b] * 64].reshape(1, h, nb[b], 64, 128).astype(np.float32)
            q8, n, m, s_, st = O.nsn_encode(x, 3)
            pages = cache.block_table[b, :nb[b]].long().cpu()
            # the block records keep K as paired halves and V as paired rows
            codes = w.from_code_order(pool["codes"][:, pages], 3, pool.get("code_order", 0))
            got = codes.cpu().numpy().reshape(-1, 3072)
            want = np.stack([O.pack3(blk) for blk in q8.reshape(-1, 64, 128)])
            assert np.array_equal(got, want), (b, kv)
            assert np.array_equal(bits16(pool["norm"][:, pages]).reshape(-1), n.view(np.uint16).reshape(-1))
            assert np.array_equal(bits16(pool["scale"][:, pages]).reshape(-1), s_.view(np.uint16).reshape(-1))
        t = (lens[b] + steps) % 64
        assert np.array_equal(cache.k_tail[b, :, :t].float().cpu().numpy(), hist_k[b][:, nb[b] * 64:].astype(np.float32))


def test_split_kv_merge_equals_one_pass():
    """cfg4-shaped (INT5, GQA 64:8) sequence split into 3 shards on one GPU."""
    from nsn_b200 import codec, kernel, workloads
    from nsn_b200.splitkv import ShardedSequence, merge_shards, shard_range
    gen = torch.Generator(device="cuda").manual_seed(4)
    h, hq, nb, t = 8, 64, 37, 64
    T = nb * 64 + t
    k = workloads.torch_kv(gen, (1, h, T, 128), workloads.K_OUTLIERS_8, 0.5)
    v = workloads.torch_kv(gen, (1, h, T, 128), (), 1.0)
    q = (torch.randn((1, hq, 1, 128), generator=gen, device="cuda") / np.sqrt(128)).half()
    g = codec.encode_group(k[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=5)
    vg = codec.encode_group(v[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 0, bits=5)
    kt, vt = k[:, :, nb * 64:].contiguous(), v[:, :, nb * 64:].contiguous()
    one = kernel.pipeline("GQA_FUSED", (g, kt, q, vg, vt)).float().reshape(hq, 128)
    world = 3
    Os, Ss = [], []
    for r in range(world):
        s, e = shard_range(nb, world, r)
        sub = lambda gr: dict(codes=gr["codes"][:, :, s:e].contiguous(),
                              metas=tuple(m[:, :, s:e].contiguous() for m in gr["metas"]))
        last = r == world - 1
        sh = ShardedSequence(sub(g), sub(vg), kt if last else None, vt if last else None, h, hq, 5)
        o, lse = sh.local(q)
        Os.append(o.clone())
        Ss.append(lse.clone())
        sh.check()
    out, status = merge_shards(torch.stack(Os), torch.stack(Ss), dtype=torch.float16)
    assert int(status.item()) == 0
    # the packed-record form (what one all-gather returns) merges to the same bits
    from nsn_b200.splitkv import merge_records
    records = torch.cat([torch.cat([o.reshape(-1), s_.reshape(-1)]) for o, s_ in zip(Os, Ss)])
    out_r, status_r = merge_records(records, world, hq, dtype=torch.float16)
    assert int(status_r.item()) == 0
    assert torch.equal(out_r.view(torch.int16), out.view(torch.int16))
    ok, err = O.within_tolerance(out.float().cpu().numpy(), one.cpu().numpy(), *O.TOLERANCE["float16"])
    assert ok, err
    # and against the oracle
    kk, vv = k.float().cpu().numpy(), v.float().cpu().numpy()
    fulls = []
    for src in (kk, vv):
        qq, n, m, s_, st = O.nsn_encode(src[:, :, :nb * 64].reshape(1, h, nb, 64, 128), 5)
        fulls.append(O.restore_full(qq, n, m, s_, src[:, :, nb * 64:], "float16"))
    want, _ = O.bridge_attention(q.float().cpu().numpy(), fulls[0], fulls[1])
    ok, err = O.within_tolerance(out.float().cpu().numpy(), want[0], *O.TOLERANCE["float16"])
    assert ok, err


def test_paged_export_import_and_bytes_round_trip():
    """A live paged cache's sequence: exported to the reference layout it attends like the
    cache (bridge arm on the exported data), and through the byte container it loads
    into a second cache with identical pages and identical attention outputs.  Reference-
    layout data with a tail of 64+ tokens is resealed on import."""
    from nsn_b200 import codec, kernel, workloads
    from nsn_b200.paged import PagedKVCache
    rng = np.random.default_rng(31)
    h, hq, lens = 2, 8, [150, 64, 97]
    cache = PagedKVCache(len(lens), h, max_blocks=6, bits=3, dtype=torch.float16, hq=hq)
    for b, L in enumerate(lens):
        cache.prefill(b, torch.from_numpy(workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5)).cuda(),
                      torch.from_numpy(workloads.np_kv(rng, (h, L, 128), (), 0.5)).cuda())
    for s in range(40):
        kn = torch.from_numpy(workloads.np_kv(rng, (len(lens), h, 1, 128), (), 0.5)[:, :, 0]).cuda()
        vn = torch.from_numpy(workloads.np_kv(rng, (len(lens), h, 1, 128), (), 0.5)[:, :, 0]).cuda()
        q = torch.from_numpy((rng.standard_normal((len(lens), hq, 128)) / np.sqrt(128)).astype(np.float16)).cuda()
        cache.step(q, kn, vn)
    cache.check()
    q = torch.from_numpy((rng.standard_normal((len(lens), hq, 128)) / np.sqrt(128)).astype(np.float16)).cuda()
    out = cache.attend(q).clone()
    cache.check()
    other = PagedKVCache(len(lens), h, max_blocks=6, bits=3, dtype=torch.float16, hq=hq)
    for b in range(len(lens)):
        kg, kt, vg, vt = cache.export_groups(b)
        want = kernel.pipeline("TORCH_SDPA", (kg, kt, q[b].reshape(1, hq, 1, 128), vg, vt)).float().reshape(hq, 128)
        ok, err = O.within_tolerance(out[b].float().cpu().numpy(), want.cpu().numpy(), *O.TOLERANCE["float16"])
        assert ok, (b, err)
        other.load_bytes(b, cache.to_bytes(b))
    assert torch.equal(other.n_blocks, cache.n_blocks) and torch.equal(other.tail_len, cache.tail_len)
    for b in range(len(lens)):
        nb, t = int(cache.n_blocks[b]), int(cache.tail_len[b])
        pages = cache.block_table[b, :nb].long()
        for pa, pb in ((cache.k_pool, other.k_pool), (cache.v_pool, other.v_pool)):
            for key in ("codes", "norm", "min", "scale"):
                assert torch.equal(pa[key][:, pages], pb[key][:, pages]), (b, key)
        assert torch.equal(cache.k_tail[b, :, :t], other.k_tail[b, :, :t])
    out2 = other.attend(q)
    other.check()
    assert torch.equal(out2.view(torch.int16), out.view(torch.int16))
    # reference layout with a 70-token tail (the reference policy keeps 64..127): resealed on import
    x = torch.from_numpy(workloads.np_kv(rng, (1, h, 3 * 64 + 70, 128), (), 0.5)).cuda()
    g = codec.encode_group(x[:, :, :192].reshape(1, h, 3, 64, 128), 0)
    third = PagedKVCache(1, h, max_blocks=6, bits=3, dtype=torch.float16, hq=hq)
    third.import_groups(0, g, x[:, :, 192:].contiguous(), g, x[:, :, 192:].contiguous())
    assert int(third.n_blocks[0]) == 4 and int(third.tail_len[0]) == 6
    g4 = codec.encode_group(x[:, :, :256].reshape(1, h, 4, 64, 128), 0)
    kg, kt, _, _ = third.export_groups(0)
    assert torch.equal(kg["codes"], g4["codes"]) and torch.equal(kg["headers"], g4["headers"])
    assert torch.equal(kt, x[:, :, 256:])


def test_full_table_row_keeps_its_tail():
    """With the plan's host check bypassed (attend + seal called directly, as a replayed
    graph would), a tail that fills when its sequence has no page left stays in place: the
    status flags NSNKV_ST_CAPACITY, the next append is attended but not stored, and the
    other sequence's pages and counters are untouched."""
    from nsn_b200 import primitives as w
    from nsn_b200 import workloads
    from nsn_b200.paged import PagedKVCache
    rng = np.random.default_rng(23)
    h, hq = 2, 8
    cache = PagedKVCache(2, h, max_blocks=2, bits=3, dtype=torch.float16, hq=hq)
    lens = [2 * 64 + 62, 64 + 6]
    for b, L in enumerate(lens):
        cache.prefill(b, torch.from_numpy(workloads.np_kv(rng, (h, L, 128), workloads.K_OUTLIERS_4, 0.5)).cuda(),
                      torch.from_numpy(workloads.np_kv(rng, (h, L, 128), (), 0.5)).cuda())
    pages1 = cache.block_table[1].long()
    before1 = cache.records[:, pages1].clone()

    def one_step():
        q = torch.from_numpy((rng.standard_normal((2, hq, 128)) / np.sqrt(128)).astype(np.float16)).cuda()
        kn = torch.from_numpy(workloads.np_kv(rng, (2, h, 1, 128), (), 0.5)[:, :, 0]).cuda()
        vn = torch.from_numpy(workloads.np_kv(rng, (2, h, 1, 128), (), 0.5)[:, :, 0]).cuda()
        out = cache.attend(q, kn, vn)
        cache.seal(1)
        return out

    one_step()  # sequence 0: tail 62 -> 63
    cache.check()
    one_step()  # tail 63 -> 64 with both pages used: no seal
    assert cache.n_blocks.cpu().tolist() == [2, 1] and cache.tail_len.cpu().tolist() == [64, 8]
    with pytest.raises(w.IntegrityError):
        cache.check()
    cache.status.zero_()
    out = one_step()  # the append to the full tail is refused, the token still attended
    assert cache.n_blocks.cpu().tolist() == [2, 1] and cache.tail_len.cpu().tolist() == [64, 9]
    one_step()  # and again: the full tail stays at its 64 rows
    assert cache.n_blocks.cpu().tolist() == [2, 1] and cache.tail_len.cpu().tolist() == [64, 10]
    with pytest.raises(w.IntegrityError):
        cache.check()
    assert torch.isfinite(out.float()).all()
    assert torch.equal(cache.records[:, pages1], before1)  # sequence 1 sealed nothing, its pages unchanged


@pytest.mark.parametrize("mode", ["exact", "k"])
def test_host_buffer_step_matches_device_step(mode):
    """nsnkv_paged_step_host (PagedKVCache.step_host) against nsnkv_paged_step on a twin
    cache: 70 steps with seals, the inputs from pinned host memory, two output slots in flight
    at once and the host reading each output only after its done event; every output and the
    final counters and records are bit-equal.  Another device plan's steps on the caller's
    stream interleave with the copies."""
    from nsn_b200 import workloads
    from nsn_b200.paged import PagedKVCache
    rng = np.random.default_rng(31)
    h, hq, lens = 2, 8, [3 * 64 + 60, 64 + 1, 5]
    caches = []
    for _ in range(2):
        c = PagedKVCache(len(lens), h, max_blocks=6, bits=3, dtype=torch.float16, hq=hq, restore_rounding=mode)
        r2 = np.random.default_rng(32)
        for b, L in enumerate(lens):
            c.prefill(b, torch.from_numpy(workloads.np_kv(r2, (h, L, 128), workloads.K_OUTLIERS_4, 0.5)).cuda(),
                      torch.from_numpy(workloads.np_kv(r2, (h, L, 128), (), 0.5)).cuda())
        caches.append(c)
    dev_cache, host_cache = caches
    B, steps = len(lens), 70
    q = (rng.standard_normal((steps, B, hq, 128)) / np.sqrt(128)).astype(np.float16)
    kn = workloads.np_kv(rng, (steps, B, h, 128), (), 0.5)
    vn = workloads.np_kv(rng, (steps, B, h, 128), (), 0.5)
    inh = torch.from_numpy(np.concatenate([q.reshape(steps, -1), kn.reshape(steps, -1), vn.reshape(steps, -1)],
                                          1)).pin_memory()
    outh = [torch.empty((B, hq, 128), dtype=torch.float16).pin_memory() for _ in range(2)]
    evs = [torch.cuda.Event() for _ in range(2)]
    got, want = [], []
    for s in range(steps):
        j = s % 2
        if s >= 2:
            evs[j].synchronize()
            got.append(outh[j].clone())
        host_cache.step_host(inh[s], outh[j], done_event=evs[j])
        want.append(dev_cache.step(torch.from_numpy(q[s]).cuda(), torch.from_numpy(kn[s]).cuda(),
                                   torch.from_numpy(vn[s]).cuda()).cpu())
    for s in range(steps - 2, steps):
        evs[s % 2].synchronize()
        got.append(outh[s % 2].clone())
    torch.cuda.synchronize()
    dev_cache.check()
    host_cache.check()
    for s in range(steps):
        assert torch.equal(got[s], want[s]), s
    assert torch.equal(dev_cache.n_blocks, host_cache.n_blocks) and torch.equal(dev_cache.tail_len,
                                                                                 host_cache.tail_len)
    assert list(dev_cache.host_blocks) == list(host_cache.host_blocks)
    assert torch.equal(dev_cache.records, host_cache.records)
    with pytest.raises(Exception):
        host_cache.step_host(inh[0].cuda(), outh[0])  # device tensors are refused
